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
   else if(mode == kSumEpi)
      k_seg_reduce< T, VB, CH, kSumEpi ><<< grid, kThreads, 0, stream >>>(p);
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
int launch_map_shape(const SegParams& p, int mode, cudaStream_t stream)
{
   const int64_t groups = (p.num_rows + 31) / 32;
   int64_t blocks = (groups * 32 + kThreads - 1) / kThreads;
   const int64_t cap = (int64_t)148 * 16;
   if(blocks > cap) blocks = cap;
   if(blocks < 1) blocks = 1;
   if(mode == kCopyLast)
      k_row_map< T, VB, CH, kCopyLast ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else if(mode == kSum)
      k_row_map< T, VB, CH, kSum ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else if(mode == kSumEpi)
      k_row_map< T, VB, CH, kSumEpi ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else if(mode == kLse)
      k_row_map< T, VB, CH, kLse ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else
      k_row_map< T, VB, CH, kLseBwd ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   return check_launch("k_row_map");
}

template < typename T, int VB, int CH >
int launch_scatter_shape(const SegParams& p, const uint32_t* cover, int64_t out_rows, cudaStream_t stream)
{
   const unsigned grid = (unsigned)((p.num_tiles * 32 + kThreads - 1) / kThreads);
   if(p.epi_div)
      k_scatter_rows< T, VB, CH, true ><<< grid, kThreads, 0, stream >>>(p);
   else
      k_scatter_rows< T, VB, CH, false ><<< grid, kThreads, 0, stream >>>(p);
   int rc = check_launch("k_scatter_rows");
   if(rc || !cover) return rc;  // no bitmap: every out row is the target of an edge
   int64_t blocks = (out_rows + kThreads - 1) / kThreads;
   const int64_t cap = (int64_t)148 * 8;
   if(blocks > cap) blocks = cap;
   if(blocks < 1) blocks = 1;
   k_zero_uncovered< T, VB, CH ><<< (unsigned)blocks, kThreads, 0, stream >>>(p, cover, out_rows);
   return check_launch("k_zero_uncovered");
}

template < typename T >
int launch_map_packed(const SegParams& p, int mode, cudaStream_t stream)
{
   const int64_t groups = (p.num_rows + 31) / 32;
   int64_t blocks = (groups * 32 + kThreads - 1) / kThreads;
   const int64_t cap = (int64_t)148 * 16;
   if(blocks > cap) blocks = cap;
   if(blocks < 1) blocks = 1;
   if(mode == kCopyLast)
      k_row_map_packed< T, kCopyLast ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else if(mode == kSum)
      k_row_map_packed< T, kSum ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else if(mode == kSumEpi)
      k_row_map_packed< T, kSumEpi ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else if(mode == kLse)
      k_row_map_packed< T, kLse ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else
      k_row_map_packed< T, kLseBwd ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   return check_launch("k_row_map_packed");
}

// The short-row kernel (returns at once unless the plan has repeated rows and
// no row above kShortRowEdges edges).
template < typename T >
int launch_rows_packed(const SegParams& p, int mode, cudaStream_t stream)
{
   const int rpi = 32 / (p.lanes > 0 ? p.lanes : 1);
   const int64_t warps = (p.num_rows + rpi - 1) / rpi;
   int64_t blocks = (warps * 32 + kThreads - 1) / kThreads;
   const int64_t cap = (int64_t)148 * 16;
   if(blocks > cap) blocks = cap;
   if(blocks < 1) blocks = 1;
   if(mode == kSum)
      k_seg_rows_packed< T, kSum ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else if(mode == kSumEpi)
      k_seg_rows_packed< T, kSumEpi ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else if(mode == kLse)
      k_seg_rows_packed< T, kLse ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   else
      k_seg_rows_packed< T, kLseBwd ><<< (unsigned)blocks, kThreads, 0, stream >>>(p);
   return check_launch("k_seg_rows_packed");
}

template < typename T >
int launch_scatter_packed(const SegParams& p, const uint32_t* cover, int64_t out_rows, cudaStream_t stream)
{
   const unsigned grid = (unsigned)((p.num_tiles * 32 + kThreads - 1) / kThreads);
   if(p.epi_div)
      k_scatter_rows_packed< T, true ><<< grid, kThreads, 0, stream >>>(p);
   else
      k_scatter_rows_packed< T, false ><<< grid, kThreads, 0, stream >>>(p);
   int rc = check_launch("k_scatter_rows_packed");
   if(rc || !cover) return rc;  // no bitmap: every out row is the target of an edge
   int64_t blocks = (out_rows + kThreads - 1) / kThreads;
   const int64_t cap = (int64_t)148 * 8;
   if(blocks > cap) blocks = cap;
   if(blocks < 1) blocks = 1;
   k_zero_uncovered< T, 16, 1 ><<< (unsigned)blocks, kThreads, 0, stream >>>(p, cover, out_rows);
   return check_launch("k_zero_uncovered");
}

template < typename T >
int launch_scatter_lse_bwd(const SegParams& p, const uint32_t* cover, int64_t out_rows, cudaStream_t stream)
{
   const unsigned grid = (unsigned)((p.num_tiles * 32 + kThreads - 1) / kThreads);
   k_scatter_lse_bwd_packed< T ><<< grid, kThreads, 0, stream >>>(p);
   int rc = check_launch("k_scatter_lse_bwd_packed");
   if(rc || !cover) return rc;  // no bitmap: every message row is used by an edge
   int64_t blocks = (out_rows + kThreads - 1) / kThreads;
   const int64_t cap = (int64_t)148 * 8;
   if(blocks > cap) blocks = cap;
   if(blocks < 1) blocks = 1;
   k_zero_uncovered< T, 16, 1 ><<< (unsigned)blocks, kThreads, 0, stream >>>(p, cover, out_rows);
   return check_launch("k_zero_uncovered");
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
int launch_row_map(const SegParams& p, int mode, int vb, int chmax, cudaStream_t stream)
{
   if(chmax == kPackedCh) return launch_map_packed< T >(p, mode, stream);
   RELM_MP_SHAPE_DISPATCH(T, launch_map_shape, p, mode, stream);
}

template < typename T >
int launch_scatter_rows(const SegParams& p, const uint32_t* cover, int64_t out_rows, int vb, int chmax,
                        cudaStream_t stream)
{
   if(chmax == kPackedCh) return launch_scatter_packed< T >(p, cover, out_rows, stream);
   RELM_MP_SHAPE_DISPATCH(T, launch_scatter_shape, p, cover, out_rows, stream);
}

template < typename T >
int launch_seg_reduce(const SegParams& pm, int vb_map, int ch_map, const SegParams& p, int vb, int chmax, int mode,
                      cudaStream_t stream)
{
   // Plans whose rows hold at most one edge are served by the row map; the
   // merge-path kernels return at once for them (and vice versa), decided on
   // the device from the plan's has_dups flag.
   int rc;
   if((pm.launch & kLaunchRowMap) && (rc = launch_row_map< T >(pm, mode, vb_map, ch_map, stream))) return rc;
   if(pm.short_rows && (pm.launch & kLaunchShort) && (rc = launch_rows_packed< T >(pm, mode, stream))) return rc;
   if(!(p.launch & kLaunchMerge)) return RELM_MP_OK;
   auto run = [&]() -> int { RELM_MP_SHAPE_DISPATCH(T, launch_reduce_shape, p, mode, stream); };
   if((rc = run())) return rc;
   if(mode == kSum) return launch_fixups< T, kSum >(p, stream);
   if(mode == kSumEpi) return launch_fixups< T, kSumEpi >(p, stream);
   if(mode == kLse) return launch_fixups< T, kLse >(p, stream);
   return launch_fixups< T, kLseBwd >(p, stream);
}

template < typename T, int PB, int MODE, bool FULL >
int launch_stream_shape(const SegParams& p, cudaStream_t stream)
{
   constexpr int NT = (MODE == kLseBwd) ? 2 : 1;
   const size_t smem = (size_t)kStreamWarps * stream_warp_bytes(NT, MODE == kSumEpi && p.epi_div);
   static bool configured = false;  // one attribute call per instantiation (per process)
   if(!configured) {
      const size_t most = (size_t)kStreamWarps * stream_warp_bytes(NT, MODE == kSumEpi);
      const int rc = check_cuda(
         cudaFuncSetAttribute(k_seg_stream< T, PB, MODE, FULL >, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)most),
         "k_seg_stream smem attribute"
      );
      if(rc) return rc;
      configured = true;
   }
   const unsigned grid = (unsigned)((p.num_tiles + kStreamWarps - 1) / kStreamWarps);
   k_seg_stream< T, PB, MODE, FULL ><<< grid, kStreamThreads, smem, stream >>>(p);
   return check_launch("k_seg_stream");
}

template < typename T, int PB, bool FULL >
int launch_stream_full(const SegParams& p, int mode, cudaStream_t stream)
{
   if(mode == kSum) return launch_stream_shape< T, PB, kSum, FULL >(p, stream);
   if(mode == kSumEpi) return launch_stream_shape< T, PB, kSumEpi, FULL >(p, stream);
   if(mode == kLse) return launch_stream_shape< T, PB, kLse, FULL >(p, stream);
   return launch_stream_shape< T, PB, kLseBwd, FULL >(p, stream);
}

// Rows of 32 * PB bytes (PB <= 16) take the FULL form of the kernel, whose
// layout constants match what the host chose for them (choose_stream_shape).
template < typename T, int PB >
int launch_stream_mode(const SegParams& p, int mode, cudaStream_t stream)
{
   if constexpr(PB <= 16) {
      constexpr int cbw = 32 * PB;
      constexpr int rows = kStreamStageBytes / cbw < 32 ? kStreamStageBytes / cbw : 32;
      if(p.lanes == 32 && p.col_blocks == 1 && p.block_cols * (int64_t)sizeof(T) == cbw && p.ch == rows &&
         p.emb * (int64_t)sizeof(T) == cbw)
         return launch_stream_full< T, PB, true >(p, mode, stream);
   }
   return launch_stream_full< T, PB, false >(p, mode, stream);
}

template < typename T >
int launch_seg_stream(const SegParams& pm, int vb_map, int ch_map, const SegParams& p, int pb, int mode,
                      cudaStream_t stream)
{
   int rc;
   if((pm.launch & kLaunchRowMap) && (rc = launch_row_map< T >(pm, mode, vb_map, ch_map, stream))) return rc;
   if(pm.short_rows && (pm.launch & kLaunchShort) && (rc = launch_rows_packed< T >(pm, mode, stream))) return rc;
   if(!(p.launch & kLaunchMerge)) return RELM_MP_OK;
   constexpr int ES = (int)sizeof(T);
   if(pb == 4 && ES <= 4) {
      rc = launch_stream_mode< T, (ES <= 4 ? 4 : 8) >(p, mode, stream);
   } else if(pb == 8) {
      rc = launch_stream_mode< T, 8 >(p, mode, stream);
   } else if(pb == 16) {
      rc = launch_stream_mode< T, 16 >(p, mode, stream);
   } else if(pb == 32) {
      rc = launch_stream_mode< T, 32 >(p, mode, stream);
   } else {
      return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported stream chunk width");
   }
   if(rc) return rc;
   if(mode == kSum) return launch_fixups< T, kSum >(p, stream);
   if(mode == kSumEpi) return launch_fixups< T, kSumEpi >(p, stream);
   if(mode == kLse) return launch_fixups< T, kLse >(p, stream);
   return launch_fixups< T, kLseBwd >(p, stream);
}

}  // namespace relm_mp

#define RELM_MP_INSTANTIATE(T)                                                                  \
   namespace relm_mp {                                                                          \
   template int launch_row_map< T >(const SegParams&, int, int, int, cudaStream_t);             \
   template int launch_scatter_rows< T >(const SegParams&, const uint32_t*, int64_t, int, int, cudaStream_t); \
   template int launch_scatter_lse_bwd< T >(const SegParams&, const uint32_t*, int64_t, cudaStream_t);        \
   template int launch_seg_reduce< T >(const SegParams&, int, int, const SegParams&, int, int, int, cudaStream_t); \
   template int launch_seg_stream< T >(const SegParams&, int, int, const SegParams&, int, int, cudaStream_t);     \
   }
