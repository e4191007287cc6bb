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
// Layout and lanes: a row of `emb` elements is covered by `lpr` lanes, each
// holding VB bytes per load (VB = 16 when the row size and pointers allow it),
// `ch` such chunks per lane; the warp works on 32 / lpr edges of the current
// row at once and folds the lane groups with shuffles at the end of the row.
// Every load is a full-width coalesced load of one gathered row; there are no
// atomics and no data-dependent waits, and the result does not depend on
// scheduling (bit-identical across runs).
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
   int64_t emb;
   int lpr;             // lanes per row (power of two <= 32)
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

template < typename T, int VB, int CH >
__global__ void __launch_bounds__(kThreads) k_gather_last(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = VB / (int)sizeof(T);
   constexpr int UR = 4;
   const int lane = threadIdx.x & 31;
   const int lpr = p.lpr;
   const int epw = 32 / lpr;
   const int grp = lane / lpr;
   const int sub = lane % lpr;
   const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
   const T* table = static_cast< const T* >(p.table);
   T* out = static_cast< T* >(p.out);
   const int64_t step = nwarps * epw * UR;
   for(int64_t base = warp * epw * UR; base < p.num_rows; base += step) {
      int64_t src[UR];
      int64_t rows[UR];
#pragma unroll
      for(int u = 0; u < UR; ++u) {
         rows[u] = base + (int64_t)u * epw + grp;
         src[u] = -1;
         if(rows[u] < p.num_rows) {
            const int32_t e1 = p.row_ptr[rows[u] + 1];
            if(e1 > p.row_ptr[rows[u]]) src[u] = p.gidx[e1 - 1];
         }
      }
      for(int cb = 0; cb < p.col_blocks; ++cb) {
         A v[UR][CH][VN];
#pragma unroll
         for(int u = 0; u < UR; ++u) {
#pragma unroll
            for(int c = 0; c < CH; ++c) {
               const int64_t col = cb * p.block_cols + (int64_t)(c * lpr + sub) * VN;
#pragma unroll
               for(int k = 0; k < VN; ++k) v[u][c][k] = A(0);
               if(c < p.ch && col < p.emb && src[u] >= 0) load_vec< T, VB >(table + src[u] * p.emb + col, v[u][c]);
            }
         }
#pragma unroll
         for(int u = 0; u < UR; ++u) {
            if(rows[u] >= p.num_rows) continue;
#pragma unroll
            for(int c = 0; c < CH; ++c) {
               const int64_t col = cb * p.block_cols + (int64_t)(c * lpr + sub) * VN;
               if(c < p.ch && col < p.emb) store_vec< T, VB >(out + rows[u] * p.emb + col, v[u][c]);
            }
         }
      }
   }
}

template < typename T, int VB, int CH, int MODE >
__global__ void __launch_bounds__(kThreads) k_seg_reduce(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = VB / (int)sizeof(T);
   constexpr int U = (VB * CH <= 8) ? 8 : ((VB * CH <= 16) ? 4 : 2);
   const int64_t tile = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   if(tile >= p.num_tiles) return;
   const int lane = threadIdx.x & 31;
   const int lpr = p.lpr;
   const int epw = 32 / lpr;
   const int grp = lane / lpr;
   const int sub = lane % lpr;
   const int r_begin = p.tile_row[tile];
   const int j_begin = p.tile_edge[tile];
   const int r_end = p.tile_row[tile + 1];
   const int j_end = p.tile_edge[tile + 1];
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
      int64_t col[CH];
      bool cv[CH];
#pragma unroll
      for(int c = 0; c < CH; ++c) {
         col[c] = cb * p.block_cols + (int64_t)(c * lpr + sub) * VN;
         cv[c] = c < p.ch && col[c] < p.emb;
      }
      int r = r_begin;
      int j = j_begin;
      while(true) {
         const bool row_ends = r < r_end;
         const int stop = row_ends ? p.row_ptr[r + 1] : j_end;
         A acc[CH][VN];
         A aux[CH][VN];
         A ownv[CH][VN];
#pragma unroll
         for(int c = 0; c < CH; ++c) {
#pragma unroll
            for(int k = 0; k < VN; ++k) {
               acc[c][k] = (MODE == kLse) ? ninf : A(0);
               aux[c][k] = A(0);
               ownv[c][k] = A(0);
            }
         }
         if(MODE == kLseBwd && j < stop) {
#pragma unroll
            for(int c = 0; c < CH; ++c)
               if(cv[c]) load_vec< T, VB >(own + (int64_t)r * p.emb + col[c], ownv[c]);
         }
         int jj = j + grp;
         for(; jj + (U - 1) * epw < stop; jj += U * epw) {
            int32_t g[U];
#pragma unroll
            for(int u = 0; u < U; ++u) g[u] = p.gidx[jj + u * epw];
            A v[U][CH][VN];
            A w[(MODE == kLseBwd) ? U : 1][CH][VN];
#pragma unroll
            for(int u = 0; u < U; ++u) {
#pragma unroll
               for(int c = 0; c < CH; ++c) {
                  if(cv[c]) {
                     load_vec< T, VB >(table + (int64_t)g[u] * p.emb + col[c], v[u][c]);
                     if(MODE == kLseBwd)
                        load_vec< T, VB >(table2 + (int64_t)g[u] * p.emb + col[c], w[(MODE == kLseBwd) ? u : 0][c]);
                  }
               }
            }
#pragma unroll
            for(int c = 0; c < CH; ++c) {
#pragma unroll
               for(int k = 0; k < VN; ++k) {
                  if(MODE == kSum) {
#pragma unroll
                     for(int u = 0; u < U; ++u) acc[c][k] += v[u][c][k];
                  } else if(MODE == kLse) {
                     A mn = acc[c][k];
#pragma unroll
                     for(int u = 0; u < U; ++u) mn = nanmax(mn, v[u][c][k]);
                     A s = aux[c][k] * exp_acc(acc[c][k] - mn);
#pragma unroll
                     for(int u = 0; u < U; ++u) s += exp_acc(v[u][c][k] - mn);
                     acc[c][k] = mn;
                     aux[c][k] = s;
                  } else {
#pragma unroll
                     for(int u = 0; u < U; ++u)
                        acc[c][k] += v[u][c][k] * exp_acc(ownv[c][k] - w[(MODE == kLseBwd) ? u : 0][c][k]);
                  }
               }
            }
         }
         for(; jj < stop; jj += epw) {
            const int32_t g = p.gidx[jj];
            A v[CH][VN];
            A w[CH][VN];
#pragma unroll
            for(int c = 0; c < CH; ++c) {
               if(cv[c]) {
                  load_vec< T, VB >(table + (int64_t)g * p.emb + col[c], v[c]);
                  if(MODE == kLseBwd) load_vec< T, VB >(table2 + (int64_t)g * p.emb + col[c], w[c]);
               }
            }
#pragma unroll
            for(int c = 0; c < CH; ++c) {
#pragma unroll
               for(int k = 0; k < VN; ++k) {
                  if(MODE == kSum) {
                     acc[c][k] += v[c][k];
                  } else if(MODE == kLse) {
                     const A mn = nanmax(acc[c][k], v[c][k]);
                     aux[c][k] = aux[c][k] * exp_acc(acc[c][k] - mn) + exp_acc(v[c][k] - mn);
                     acc[c][k] = mn;
                  } else {
                     acc[c][k] += v[c][k] * exp_acc(ownv[c][k] - w[c][k]);
                  }
               }
            }
         }
         // Fold the lane groups (each holds a strided subset of the row's edges).
         for(int off = lpr; off < 32; off <<= 1) {
#pragma unroll
            for(int c = 0; c < CH; ++c) {
#pragma unroll
               for(int k = 0; k < VN; ++k) {
                  const A o = __shfl_xor_sync(0xffffffffu, acc[c][k], off);
                  if(MODE == kLse) {
                     const A oa = __shfl_xor_sync(0xffffffffu, aux[c][k], off);
                     lse_merge(acc[c][k], aux[c][k], o, oa);
                  } else {
                     acc[c][k] += o;
                  }
               }
            }
         }
         if(row_ends) {
            const bool began_before = (r == r_begin) && (p.row_ptr[r] < j_begin);
            if(grp == 0) {
#pragma unroll
               for(int c = 0; c < CH; ++c) {
                  if(!cv[c]) continue;
                  if(began_before) {
                     const int64_t off = tile * p.emb + col[c];
#pragma unroll
                     for(int k = 0; k < VN; ++k) {
                        head_val[off + k] = acc[c][k];
                        if(MODE == kLse) head_aux[off + k] = aux[c][k];
                     }
                  } else {
                     A fin[VN];
#pragma unroll
                     for(int k = 0; k < VN; ++k)
                        fin[k] = (MODE == kLse) ? log_acc(aux[c][k]) + acc[c][k] : acc[c][k];
                     store_vec< T, VB >(out + (int64_t)r * p.emb + col[c], fin);
                  }
               }
            }
            if(began_before) head_row = r;
            j = stop;
            ++r;
         } else {
            if(j < stop) {
               if(grp == 0) {
#pragma unroll
                  for(int c = 0; c < CH; ++c) {
                     if(!cv[c]) continue;
                     const int64_t off = tile * p.emb + col[c];
#pragma unroll
                     for(int k = 0; k < VN; ++k) {
                        tail_val[off + k] = acc[c][k];
                        if(MODE == kLse) tail_aux[off + k] = aux[c][k];
                     }
                  }
               }
               tail_row = r;
            }
            break;
         }
      }
   }
   if(lane == 0) {
      p.head_row[tile] = head_row;
      p.tail_row[tile] = tail_row;
   }
}

template < typename T, int MODE >
__device__ __forceinline__ void fixup_combine(const SegParams& p, int64_t R, int64_t t_first, int64_t t_last,
                                              int64_t col, typename AccOf< T >::type& m,
                                              typename AccOf< T >::type& s)
{
   using A = typename AccOf< T >::type;
   const A* tail_val = static_cast< const A* >(p.tail_val);
   const A* tail_aux = static_cast< const A* >(p.tail_aux);
   for(int64_t u = t_first; u < t_last; ++u) {
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

// Warp per tile: finishes the row whose tail part is in this tile, adding the
// partials of the tiles it spans, in tile order.
template < typename T, int MODE >
__global__ void __launch_bounds__(kThreads) k_fixup(SegParams p)
{
   using A = typename AccOf< T >::type;
   const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   if(t >= p.num_tiles) return;
   const int lane = threadIdx.x & 31;
   const int R = p.head_row[t];
   if(R < 0) return;
   const int64_t t_first = ((int64_t)p.row_ptr[R] + R) / kTileItems;
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
      fixup_combine< T, MODE >(p, R, t_first, t, col, m, s);
      fixup_finish< T, MODE >(p, R, t, col, m, s);
   }
}

// Block per long row: the 8 warps each combine one contiguous slice of the
// row's partials, then warp 0 combines the 8 slice results in order.
template < typename T, int MODE >
__global__ void __launch_bounds__(kThreads) k_fixup_long(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int W = kThreads / 32;
   __shared__ A sm_m[W][32];
   __shared__ A sm_s[W][32];
   const int64_t b = blockIdx.x;
   const int count = *p.long_count;
   if(b >= count || b >= p.max_long) return;
   const int64_t t = p.long_list[b];
   const int R = p.head_row[t];
   const int64_t t_first = ((int64_t)p.row_ptr[R] + R) / kTileItems;
   const int64_t n = t - t_first;
   const int warp = threadIdx.x >> 5;
   const int lane = threadIdx.x & 31;
   const int64_t per = (n + W - 1) / W;
   const int64_t u0 = t_first + per * warp;
   const int64_t u1 = (u0 + per < t) ? u0 + per : t;
   for(int64_t col0 = 0; col0 < p.emb; col0 += 32) {
      const int64_t col = col0 + lane;
      A m = (MODE == kLse) ? -(A)INFINITY : A(0);
      A s = A(0);
      if(col < p.emb && u0 < u1) fixup_combine< T, MODE >(p, R, u0, u1, col, m, s);
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
