// Segment kernels over a plan (CSR of output rows):
//   k_gather_last - out[r] = table[gidx[last edge of r]] (fanout forward)
//   k_seg_reduce  - merge-path segment reduction, one warp per tile, with
//                   partials for rows that cross tile boundaries
//                   (SUM: fanin sum forward, both sum backwards;
//                    LSE: fanin logsumexp forward, online max / sum-exp;
//                    LSE_BWD: fanin logsumexp backward)
//   k_fixup       - combines the partials of a row in tile order (warp per row)
//   k_fixup_long  - same for rows spanning many tiles (block per row)
//
// Layout and lanes: one warp load moves one gathered row: `lanes` lanes hold
// VB bytes each (VB = row bytes / 32 rounded to a vector width the row size
// and pointers allow), wider rows take `ch` chunks per lane and very wide rows
// several column blocks. Every load is a coalesced load of one gathered row;
// there are no atomics on values and no data-dependent waits, and the result
// does not depend on scheduling (bit-identical across runs).
#pragma once

#include <math.h>

#include "relm_mp_internal.cuh"

namespace relm_mp {

enum SegMode : int { kSum = 0, kLse = 1, kLseBwd = 2 };

template < typename T >
struct AccOf {
   using type = float;
};
template <>
struct AccOf< double > {
   using type = double;
};

template < int VB >
struct Raw;
template <>
struct Raw< 2 > {
   using type = unsigned short;
};
template <>
struct Raw< 4 > {
   using type = unsigned int;
};
template <>
struct Raw< 8 > {
   using type = uint2;
};
template <>
struct Raw< 16 > {
   using type = uint4;
};

__device__ __forceinline__ float to_acc(float v) { return v; }
__device__ __forceinline__ double to_acc(double v) { return v; }
__device__ __forceinline__ float to_acc(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_acc(__half v) { return __half2float(v); }

template < typename T >
__device__ __forceinline__ T from_acc(typename AccOf< T >::type v);
template <>
__device__ __forceinline__ float from_acc< float >(float v)
{
   return v;
}
template <>
__device__ __forceinline__ double from_acc< double >(double v)
{
   return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_acc< __nv_bfloat16 >(float v)
{
   return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_acc< __half >(float v)
{
   return __float2half_rn(v);
}

template < typename T, int VB >
__device__ __forceinline__ void load_vec(const T* p, typename AccOf< T >::type (&out)[VB / sizeof(T)])
{
   using R = typename Raw< VB >::type;
   const R r = __ldg(reinterpret_cast< const R* >(p));
   const T* e = reinterpret_cast< const T* >(&r);
#pragma unroll
   for(int i = 0; i < (int)(VB / sizeof(T)); ++i) out[i] = to_acc(e[i]);
}

template < typename T, int VB >
__device__ __forceinline__ void store_vec(T* p, const typename AccOf< T >::type (&in)[VB / sizeof(T)])
{
   using R = typename Raw< VB >::type;
   R r;
   T* e = reinterpret_cast< T* >(&r);
#pragma unroll
   for(int i = 0; i < (int)(VB / sizeof(T)); ++i) e[i] = from_acc< T >(in[i]);
   *reinterpret_cast< R* >(p) = r;
}

__device__ __forceinline__ float nanmax(float a, float b) { return (a != a || a > b) ? a : b; }
__device__ __forceinline__ double nanmax(double a, double b) { return (a != a || a > b) ? a : b; }
__device__ __forceinline__ float exp_acc(float v) { return expf(v); }
__device__ __forceinline__ double exp_acc(double v) { return exp(v); }
__device__ __forceinline__ float log_acc(float v) { return logf(v); }
__device__ __forceinline__ double log_acc(double v) { return log(v); }

// (m, s) of a running log-sum-exp: value = log(s) + m. The empty state is
// (-inf, 0); a state that saw only -inf values has s = NaN, which is what the
// reference's exp(-inf - (-inf)) gives.
template < typename A >
__device__ __forceinline__ bool lse_empty(A m, A s)
{
   return s == A(0) && m == -(A)INFINITY;
}

template < typename A >
__device__ __forceinline__ void lse_merge(A& m, A& s, A m2, A s2)
{
   if(lse_empty(m2, s2)) return;
   if(lse_empty(m, s)) {
      m = m2;
      s = s2;
      return;
   }
   const A mn = nanmax(m, m2);
   s = s * exp_acc(m - mn) + s2 * exp_acc(m2 - mn);
   m = mn;
}

struct SegParams {
   const int32_t* row_ptr;
   const int32_t* gidx;
   const int32_t* tile_row;
   const int32_t* tile_edge;
   int64_t num_tiles;
   int64_t num_rows;
   int64_t num_edges;
   int tile_items;
   int64_t emb;
   int lanes;           // lanes holding a VB chunk of the row (<= 32)
   int ch;              // VB-chunks per lane in one column block (<= CH)
   int col_blocks;      // column blocks covering emb
   int64_t block_cols;  // elements per column block
   const void* table;   // gathered rows (SUM / LSE values, LSE_BWD grad_out)
   const void* table2;  // LSE_BWD: gathered logsumexp output rows
   const void* own;     // LSE_BWD: rel rows indexed by the output row
   void* out;
   void* head_val;      // [num_tiles, emb] accumulator partials (LSE: running max)
   void* tail_val;
   void* head_aux;      // LSE: running sum-exp partials
   void* tail_aux;
   int32_t* head_row;   // row whose last part is in this tile but began earlier, or -1
   int32_t* tail_row;   // row that continues past this tile, or -1
   int32_t* long_count;
   int32_t* long_list;
   int64_t max_long;
};

// Entries of gidx / row ends a warp stages in shared memory at a time.
constexpr int kStage = 256;
constexpr int kWarps = kThreads / 32;

// Column layout of one lane: chunk c covers elements [col(c), col(c) + VN).
template < int CH >
struct Cols {
   int64_t col[CH];
   bool ok[CH];
   __device__ __forceinline__ Cols(const SegParams& p, int cb, int lane, int vn)
   {
#pragma unroll
      for(int c = 0; c < CH; ++c) {
         col[c] = cb * p.block_cols + (int64_t)(c * 32 + lane) * vn;
         ok[c] = c < p.ch && lane < p.lanes && col[c] < p.emb;
      }
   }
};

// fanout forward: out[r] = table[gidx[last edge of r]], 0 for rows without
// edges. A warp owns groups of 32 consecutive rows: the lanes fetch the
// group's row_ptr / gidx entries with coalesced loads (prefetched one group
// ahead), then the whole warp copies one row per load, U rows in flight.
template < typename T, int VB, int CH >
__global__ void __launch_bounds__(kThreads) k_gather_last(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = VB / (int)sizeof(T);
   constexpr int U = (VB * CH <= 16) ? 8 : 4;
   const int lane = threadIdx.x & 31;
   const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
   const T* table = static_cast< const T* >(p.table);
   T* out = static_cast< T* >(p.out);
   const int64_t groups = (p.num_rows + 31) / 32;

   auto fetch_src = [&](int64_t g) -> int32_t {
      const int64_t r = g * 32 + lane;
      int32_t src = -1;
      if(g < groups && r < p.num_rows) {
         const int32_t e0 = p.row_ptr[r];
         const int32_t e1 = p.row_ptr[r + 1];
         if(e1 > e0) src = p.gidx[e1 - 1];
      }
      return src;
   };

   int64_t g = warp;
   int32_t src_cur = fetch_src(g);
   for(; g < groups; g += nwarps) {
      const int32_t src_next = fetch_src(g + nwarps);
      const int64_t r0 = g * 32;
      const int nrows = (int)((p.num_rows - r0) < 32 ? (p.num_rows - r0) : 32);
      for(int cb = 0; cb < p.col_blocks; ++cb) {
         const Cols< CH > cols(p, cb, lane, VN);
         for(int base = 0; base < nrows; base += U) {
            A v[U][CH][VN];
#pragma unroll
            for(int u = 0; u < U; ++u) {
               const int32_t src = __shfl_sync(0xffffffffu, src_cur, (base + u) & 31);
#pragma unroll
               for(int c = 0; c < CH; ++c) {
#pragma unroll
                  for(int k = 0; k < VN; ++k) v[u][c][k] = A(0);
                  if(base + u < nrows && src >= 0 && cols.ok[c])
                     load_vec< T, VB >(table + (int64_t)src * p.emb + cols.col[c], v[u][c]);
               }
            }
#pragma unroll
            for(int u = 0; u < U; ++u) {
               if(base + u >= nrows) break;
#pragma unroll
               for(int c = 0; c < CH; ++c)
                  if(cols.ok[c]) store_vec< T, VB >(out + (r0 + base + u) * p.emb + cols.col[c], v[u][c]);
            }
         }
      }
      src_cur = src_next;
   }
}

// Segment reduction over one merge-path tile per warp.
//
// The tile's edges are consumed as one stream, U at a time, whatever the row
// lengths: the warp first resolves the row of each of the next U edges from
// the staged row ends (shared memory), issues the U gathered row loads (one
// full row per warp load), then folds them into the running accumulator,
// finishing rows as the stream crosses their ends. Rows that began in an
// earlier tile are written as a head partial, the row still open at the end of
// the tile as a tail partial; k_fixup combines them in tile order.
template < typename T, int VB, int CH, int MODE >
__global__ void __launch_bounds__(kThreads) k_seg_reduce(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = VB / (int)sizeof(T);
   constexpr int U = (MODE == kLseBwd) ? ((VB * CH <= 16) ? 4 : 2) : ((VB * CH <= 16) ? 8 : 4);
   __shared__ int32_t s_gidx[kWarps][kStage];
   __shared__ int32_t s_rend[kWarps][kStage];
   const int wib = threadIdx.x >> 5;
   const int64_t tile = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   if(tile >= p.num_tiles) return;
   const int lane = threadIdx.x & 31;
   int32_t* sg = s_gidx[wib];
   int32_t* sr = s_rend[wib];
   const int r_begin = p.tile_row[tile];
   const int j_begin = p.tile_edge[tile];
   const int r_end = p.tile_row[tile + 1];
   const int j_end = p.tile_edge[tile + 1];
   const bool began_before = p.row_ptr[r_begin] < j_begin;
   const T* table = static_cast< const T* >(p.table);
   const T* table2 = static_cast< const T* >(p.table2);
   const T* own = static_cast< const T* >(p.own);
   T* out = static_cast< T* >(p.out);
   A* head_val = static_cast< A* >(p.head_val);
   A* tail_val = static_cast< A* >(p.tail_val);
   A* head_aux = static_cast< A* >(p.head_aux);
   A* tail_aux = static_cast< A* >(p.tail_aux);
   const A ninf = -(A)INFINITY;
   int head_row = -1;
   int tail_row = -1;

   for(int cb = 0; cb < p.col_blocks; ++cb) {
      const Cols< CH > cols(p, cb, lane, VN);
      int gbase = j_begin, gcount = 0;
      int rbase = r_begin, rcount = 0;
      // End (exclusive edge index) of row R < r_end, from the staged row ends.
      auto row_end = [&](int R) -> int {
         if(R - rbase >= rcount) {
            __syncwarp();
            rbase = R;
            rcount = (r_end - R) < kStage ? (r_end - R) : kStage;
            for(int i = lane; i < rcount; i += 32) sr[i] = p.row_ptr[R + 1 + i];
            __syncwarp();
         }
         return sr[R - rbase];
      };
      A acc[CH][VN];
      A aux[CH][VN];
      auto reset = [&]() {
#pragma unroll
         for(int c = 0; c < CH; ++c)
#pragma unroll
            for(int k = 0; k < VN; ++k) {
               acc[c][k] = (MODE == kLse) ? ninf : A(0);
               aux[c][k] = A(0);
            }
      };
      // Finishes row R: final output, or the head partial when it began earlier.
      auto flush = [&](int R) {
         const bool head = (R == r_begin) && began_before;
#pragma unroll
         for(int c = 0; c < CH; ++c) {
            if(!cols.ok[c]) continue;
            if(head) {
               const int64_t off = tile * p.emb + cols.col[c];
#pragma unroll
               for(int k = 0; k < VN; ++k) {
                  head_val[off + k] = acc[c][k];
                  if(MODE == kLse) head_aux[off + k] = aux[c][k];
               }
            } else {
               A fin[VN];
#pragma unroll
               for(int k = 0; k < VN; ++k) fin[k] = (MODE == kLse) ? log_acc(aux[c][k]) + acc[c][k] : acc[c][k];
               store_vec< T, VB >(out + (int64_t)R * p.emb + cols.col[c], fin);
            }
         }
         if(head) head_row = R;
         reset();
      };

      reset();
      int R = r_begin;   // next row to finish
      int Rw = r_begin;  // row of the next edge
      int rend_w = (Rw < r_end) ? row_end(Rw) : INT_MAX;
      int pending = 0;   // edges folded into acc since the last flush
      for(int j = j_begin; j < j_end; j += U) {
         const int nb = (j_end - j) < U ? (j_end - j) : U;
         if(j + nb > gbase + gcount) {
            __syncwarp();
            gbase = j;
            gcount = (j_end - j) < kStage ? (j_end - j) : kStage;
            for(int i = lane; i < gcount; i += 32) sg[i] = p.gidx[j + i];
            __syncwarp();
         }
         int rr[U];
#pragma unroll
         for(int u = 0; u < U; ++u) {
            rr[u] = Rw;
            if(u < nb) {
               while(rend_w <= j + u) {
                  ++Rw;
                  rend_w = (Rw < r_end) ? row_end(Rw) : INT_MAX;
               }
               rr[u] = Rw;
            }
         }
         A v[U][CH][VN];
         A w[(MODE == kLseBwd) ? U : 1][CH][VN];
         A o[(MODE == kLseBwd) ? U : 1][CH][VN];
#pragma unroll
         for(int u = 0; u < U; ++u) {
            const int32_t g = (u < nb) ? sg[j + u - gbase] : 0;
#pragma unroll
            for(int c = 0; c < CH; ++c) {
               if(u < nb && cols.ok[c]) {
                  load_vec< T, VB >(table + (int64_t)g * p.emb + cols.col[c], v[u][c]);
                  if(MODE == kLseBwd) {
                     load_vec< T, VB >(table2 + (int64_t)g * p.emb + cols.col[c], w[(MODE == kLseBwd) ? u : 0][c]);
                     load_vec< T, VB >(own + (int64_t)rr[u] * p.emb + cols.col[c], o[(MODE == kLseBwd) ? u : 0][c]);
                  }
               }
            }
         }
#pragma unroll
         for(int u = 0; u < U; ++u) {
            if(u >= nb) break;
            while(R < rr[u]) {
               flush(R);
               pending = 0;
               ++R;
            }
            ++pending;
#pragma unroll
            for(int c = 0; c < CH; ++c) {
               if(!cols.ok[c]) continue;
#pragma unroll
               for(int k = 0; k < VN; ++k) {
                  if(MODE == kSum) {
                     acc[c][k] += v[u][c][k];
                  } else if(MODE == kLse) {
                     const A mn = nanmax(acc[c][k], v[u][c][k]);
                     aux[c][k] = aux[c][k] * exp_acc(acc[c][k] - mn) + exp_acc(v[u][c][k] - mn);
                     acc[c][k] = mn;
                  } else {
                     const int ui = (MODE == kLseBwd) ? u : 0;
                     acc[c][k] += v[u][c][k] * exp_acc(o[ui][c][k] - w[ui][c][k]);
                  }
               }
            }
         }
      }
      while(R < r_end) {
         flush(R);
         pending = 0;
         ++R;
      }
      if(pending > 0) {
#pragma unroll
         for(int c = 0; c < CH; ++c) {
            if(!cols.ok[c]) continue;
            const int64_t off = tile * p.emb + cols.col[c];
#pragma unroll
            for(int k = 0; k < VN; ++k) {
               tail_val[off + k] = acc[c][k];
               if(MODE == kLse) tail_aux[off + k] = aux[c][k];
            }
         }
         tail_row = r_end;
      }
      __syncwarp();
   }
   if(lane == 0) {
      p.head_row[tile] = head_row;
      p.tail_row[tile] = tail_row;
   }
}

// Folds tail partials [t_first, t_last) of one row into (m, s) in tile order;
// eight independent loads in flight.
template < typename T, int MODE >
__device__ __forceinline__ void fixup_combine(const SegParams& p, int64_t t_first, int64_t t_last, int64_t col,
                                              typename AccOf< T >::type& m, typename AccOf< T >::type& s)
{
   using A = typename AccOf< T >::type;
   constexpr int F = 8;
   const A* tail_val = static_cast< const A* >(p.tail_val);
   const A* tail_aux = static_cast< const A* >(p.tail_aux);
   int64_t u = t_first;
   for(; u + F <= t_last; u += F) {
      A a[F], b[F];
#pragma unroll
      for(int i = 0; i < F; ++i) {
         a[i] = tail_val[(u + i) * p.emb + col];
         b[i] = (MODE == kLse) ? tail_aux[(u + i) * p.emb + col] : A(0);
      }
#pragma unroll
      for(int i = 0; i < F; ++i) {
         if(MODE == kLse)
            lse_merge(m, s, a[i], b[i]);
         else
            m += a[i];
      }
   }
   for(; u < t_last; ++u) {
      const int64_t off = u * p.emb + col;
      if(MODE == kLse)
         lse_merge(m, s, tail_val[off], tail_aux[off]);
      else
         m += tail_val[off];
   }
}

template < typename T, int MODE >
__device__ __forceinline__ void fixup_finish(const SegParams& p, int64_t R, int64_t t, int64_t col,
                                             typename AccOf< T >::type m, typename AccOf< T >::type s)
{
   using A = typename AccOf< T >::type;
   const A* head_val = static_cast< const A* >(p.head_val);
   const A* head_aux = static_cast< const A* >(p.head_aux);
   const int64_t off = t * p.emb + col;
   A res;
   if(MODE == kLse) {
      lse_merge(m, s, head_val[off], head_aux[off]);
      res = log_acc(s) + m;
   } else {
      res = m + head_val[off];
   }
   static_cast< T* >(p.out)[R * p.emb + col] = from_acc< T >(res);
}

// Warp per tile: finishes the row whose last part is in this tile, adding the
// partials of the tiles it spans in tile order. The first tile of row R is the
// one holding its first edge, merge-path item row_ptr[R] + R.
template < typename T, int MODE >
__global__ void __launch_bounds__(kThreads) k_fixup(SegParams p)
{
   using A = typename AccOf< T >::type;
   const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   if(t >= p.num_tiles) return;
   const int lane = threadIdx.x & 31;
   const int R = p.head_row[t];
   if(R < 0) return;
   const int64_t t_first = ((int64_t)p.row_ptr[R] + R) / p.tile_items;
   if(t - t_first > kLongRowTiles) {
      if(lane == 0) {
         const int slot = atomicAdd(p.long_count, 1);
         if(slot < p.max_long) p.long_list[slot] = (int32_t)t;
      }
      return;
   }
   for(int64_t col = lane; col < p.emb; col += 32) {
      A m = (MODE == kLse) ? -(A)INFINITY : A(0);
      A s = A(0);
      fixup_combine< T, MODE >(p, t_first, t, col, m, s);
      fixup_finish< T, MODE >(p, R, t, col, m, s);
   }
}

constexpr int kLongThreads = 1024;

// Block per long row: each of the 32 warps folds one contiguous slice of the
// row's partials, then warp 0 folds the 32 slice results in order.
template < typename T, int MODE >
__global__ void __launch_bounds__(kLongThreads) k_fixup_long(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int W = kLongThreads / 32;
   __shared__ A sm_m[W][32];
   __shared__ A sm_s[W][32];
   const int64_t b = blockIdx.x;
   const int count = *p.long_count;
   if(b >= count || b >= p.max_long) return;
   const int64_t t = p.long_list[b];
   const int R = p.head_row[t];
   const int64_t t_first = ((int64_t)p.row_ptr[R] + R) / p.tile_items;
   const int64_t n = t - t_first;
   const int warp = threadIdx.x >> 5;
   const int lane = threadIdx.x & 31;
   const int64_t per = (n + W - 1) / W;
   const int64_t u0 = t_first + per * warp < t ? t_first + per * warp : t;
   const int64_t u1 = (u0 + per < t) ? u0 + per : t;
   for(int64_t col0 = 0; col0 < p.emb; col0 += 32) {
      const int64_t col = col0 + lane;
      A m = (MODE == kLse) ? -(A)INFINITY : A(0);
      A s = A(0);
      if(col < p.emb && u0 < u1) fixup_combine< T, MODE >(p, u0, u1, col, m, s);
      sm_m[warp][lane] = m;
      sm_s[warp][lane] = s;
      __syncthreads();
      if(warp == 0 && col < p.emb) {
         A mm = sm_m[0][lane];
         A ss = sm_s[0][lane];
         for(int w = 1; w < W; ++w) {
            if(MODE == kLse)
               lse_merge(mm, ss, sm_m[w][lane], sm_s[w][lane]);
            else
               mm += sm_m[w][lane];
         }
         fixup_finish< T, MODE >(p, R, t, col, mm, ss);
      }
      __syncthreads();
   }
}

// Launchers, one set per storage type (instantiated in relm_mp_seg_<dtype>.cu).
template < typename T >
int launch_gather_last(const SegParams& p, int vb, int chmax, cudaStream_t stream);
template < typename T >
int launch_seg_reduce(const SegParams& p, int mode, int vb, int chmax, cudaStream_t stream);

}  // namespace relm_mp
