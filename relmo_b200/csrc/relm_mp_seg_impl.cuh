// Launcher definitions for one storage type; included by relm_mp_seg_<dtype>.cu.
#pragma once

#include "relm_mp_segment.cuh"

namespace relm_mp {

template < typename T, int VB, int CH >
int launch_reduce_shape(const SegParams& p, int mode, cudaStream_t stream)
{
   const unsigned grid = (unsigned)((p.num_tiles * 32 + kThreads - 1) / kThreads);
   if(mode == kSum)
      k_seg_reduce< T, VB, CH, kSum ><<< grid, kThreads, 0, stream >>>(p);
   else if(mode == kLse)
      k_seg_reduce< T, VB, CH, kLse ><<< grid, kThreads, 0, stream >>>(p);
   else
      k_seg_reduce< T, VB, CH, kLseBwd ><<< grid, kThreads, 0, stream >>>(p);
   return check_launch("k_seg_reduce");
}

template < typename T, int MODE >
int launch_fixups(const SegParams& p, cudaStream_t stream)
{
   const unsigned grid = (unsigned)((p.num_tiles * 32 + kThreads - 1) / kThreads);
   k_fixup< T, MODE ><<< grid, kThreads, 0, stream >>>(p);
   int rc = check_launch("k_fixup");
   if(rc) return rc;
   if(p.max_long > 0) {
      k_fixup_long< T, MODE ><<< (unsigned)p.max_long, kLongThreads, 0, stream >>>(p);
      rc = check_launch("k_fixup_long");
   }
   return rc;
}

template < typename T, int VB, int CH >
int launch_gather_shape(const SegParams& p, cudaStream_t stream)
{
   const int64_t groups = (p.num_rows + 31) / 32;
   int64_t blocks = (groups * 32 + kThreads - 1) / kThreads;
   const int64_t cap = (int64_t)148 * 16;
   if(blocks > cap) blocks = cap;
   if(blocks < 1) blocks = 1;
   k_gather_last< T, VB, CH ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   return check_launch("k_gather_last");
}

// VB choices per storage type: the element size (scalar path) and 16 bytes are
// available with 1 or 4 chunks per lane; intermediate widths with 1 chunk.
#define RELM_MP_SHAPE_DISPATCH(T, FN, ...)                                        \
   do {                                                                            \
      constexpr int ES = (int)sizeof(T);                                           \
      if(vb == 16 && chmax == 4) return FN< T, 16, 4 >(__VA_ARGS__);               \
      if(vb == 16) return FN< T, 16, 1 >(__VA_ARGS__);                             \
      if(vb == ES && chmax == 4) return FN< T, ES, 4 >(__VA_ARGS__);               \
      if(vb == ES) return FN< T, ES, 1 >(__VA_ARGS__);                             \
      if constexpr(ES < 8) {                                                       \
         if(vb == 8) return FN< T, (ES < 8 ? 8 : 16), 1 >(__VA_ARGS__);            \
      }                                                                            \
      if constexpr(ES < 4) {                                                       \
         if(vb == 4) return FN< T, (ES < 4 ? 4 : 16), 1 >(__VA_ARGS__);            \
      }                                                                            \
      return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported vector width");           \
   } while(0)

template < typename T >
int launch_gather_last(const SegParams& p, int vb, int chmax, cudaStream_t stream)
{
   RELM_MP_SHAPE_DISPATCH(T, launch_gather_shape, p, stream);
}

template < typename T >
int launch_seg_reduce(const SegParams& p, int mode, int vb, int chmax, cudaStream_t stream)
{
   int rc;
   auto run = [&]() -> int { RELM_MP_SHAPE_DISPATCH(T, launch_reduce_shape, p, mode, stream); };
   if((rc = run())) return rc;
   if(mode == kSum) return launch_fixups< T, kSum >(p, stream);
   if(mode == kLse) return launch_fixups< T, kLse >(p, stream);
   return launch_fixups< T, kLseBwd >(p, stream);
}

}  // namespace relm_mp

#define RELM_MP_INSTANTIATE(T)                                                                  \
   namespace relm_mp {                                                                          \
   template int launch_gather_last< T >(const SegParams&, int, int, cudaStream_t);              \
   template int launch_seg_reduce< T >(const SegParams&, int, int, int, cudaStream_t);          \
   }
