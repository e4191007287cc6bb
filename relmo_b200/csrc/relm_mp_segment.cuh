// Segment kernels over a plan (CSR of output rows):
//   k_row_map     - one gathered row per output row: fanout forward, and the
//                   reductions of plans whose rows hold at most one edge
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

#include <cstring>
#include <type_traits>

#include "relm_mp_internal.cuh"

namespace relm_mp {

enum SegMode : int { kSum = 0, kLse = 1, kLseBwd = 2, kCopyLast = 3, kSumEpi = 4 };
// Kernel families a planned reduction launches (SegParams::launch).
enum LaunchFamily : int { kLaunchRowMap = 1, kLaunchShort = 2, kLaunchMerge = 4, kLaunchAll = 7 };

// kSumEpi: kSum with the epilogue of SegParams::epi_* applied where a row's
// final value is written (a separate instantiation, so kSum keeps its code).
__host__ __device__ constexpr bool sum_mode(int m) { return m == kSum || m == kSumEpi; }

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

__device__ __forceinline__ float nanmax(float a, float b)
{
   float r;
   asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
   return r;
}
__device__ __forceinline__ double nanmax(double a, double b) { return (a != a || a > b) ? a : b; }
// e^x = 2^(x * log2(e)); base-2 exponential of the hardware (ex2.approx.ftz:
// about 2 ulp, results below 2^-126 flush to zero, which only drops terms far
// below the sum they are added to).
constexpr double kLog2E = 1.4426950408889634073599246810019;
__device__ __forceinline__ float exp2_fast(float x)
{
   float r;
   asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
   return r;
}
__device__ __forceinline__ double exp2_fast(double x) { return exp2(x); }
// e^(beta * v) = 2^(v * k) with k = beta * log2(e) (LseForm::k).
__device__ __forceinline__ float exp_k(float v, float k) { return exp2_fast(v * k); }
__device__ __forceinline__ double exp_k(double v, double k) { return exp2_fast(v * k); }
__device__ __forceinline__ float log_acc(float v) { return logf(v); }
__device__ __forceinline__ double log_acc(double v) { return log(v); }

// The two logsumexp forms the kernels compute, as runtime constants:
//   plain    (fanin_reduce mode 1): m + log(sum e^(x - m)); k = log2(e),
//            eps = 0, inv_beta = 1, rows without values -inf;
//   smoothed (relmo's LogSumExpAggregation, models/aggr.py:103-123):
//            m + (1/beta) log(eps + sum e^(beta (x - m))); k = beta log2(e),
//            rows without values (1/beta) log(eps).
// The running maximum m stays in the units of x, so the smoothed form costs
// no instruction more than the plain one in the folds.
template < typename A >
struct LseForm {
   A k;
   A eps;
   A inv_beta;
   A empty;
};

// Running log-sum-exp (m, s), value = m + log(s):
//   m  running maximum, NaN as soon as a NaN was seen
//   s  sum of exp(x - m); NaN once a NaN or +inf value was seen (exp(inf - inf)
//      is NaN in the reference too)
// and, when nothing but -inf has been seen (m = -inf, s = 0), the sign of the
// zero tells "no value" (+0 -> -inf) from "only -inf values" (-0 -> NaN, the
// reference's exp(-inf - (-inf))). A block of -inf values inside a row with
// finite values therefore merges as the zero contribution it is.
template < typename A >
__device__ __forceinline__ A lse_value(A m, A s, const LseForm< A >& f)
{
   if(m == -(A)INFINITY && s == A(0)) return signbit(s) ? (A)NAN : f.empty;
   return log_acc(s + f.eps) * f.inv_beta + m;  // plain: log(s) + m exactly
}

template < typename A >
__device__ __forceinline__ void lse_merge(A& m, A& s, A m2, A s2, A k)
{
   if(m2 == -(A)INFINITY && s2 == A(0)) {
      if(signbit(s2) && m == -(A)INFINITY && s == A(0)) s = -A(0);
      return;
   }
   if(m == -(A)INFINITY && s == A(0)) {
      m = m2;
      s = s2;
      return;
   }
   const A mn = nanmax(m, m2);
   s = s * exp_k(m - mn, k) + s2 * exp_k(m2 - mn, k);
   m = mn;
}

// Folds n <= N values into (m, s): one max, one rescale of s and one
// exponential per value, all as selects (no divergence between lanes). The
// max and the sum of the exponentials are balanced trees: their dependency
// chains are log2(N) deep instead of N, which the latency-bound stream kernel
// notices more than the instruction count.
template < typename A, int N >
__device__ __forceinline__ void lse_fold(A& m, A& s, const A (&v)[N], int n, A k)
{
   A t[N];
#pragma unroll
   for(int i = 0; i < N; ++i) t[i] = (i < n) ? v[i] : -(A)INFINITY;
#pragma unroll
   for(int w = 1; w < N; w <<= 1)
#pragma unroll
      for(int i = 0; i + w < N; i += 2 * w) t[i] = nanmax(t[i], t[i + w]);
   const A mr = nanmax(m, t[0]);
   // (x - mr) is exact for the maximum itself, so a row's largest value
   // contributes exactly 1 and a single-value row returns that value.
   A e[N];
#pragma unroll
   for(int i = 0; i < N; ++i) e[i] = (i < n) ? exp_k(v[i] - mr, k) : A(0);
#pragma unroll
   for(int w = 1; w < N; w <<= 1)
#pragma unroll
      for(int i = 0; i + w < N; i += 2 * w) e[i] += e[i + w];
   const A t_sum = s * exp_k(m - mr, k) + e[0];
   const bool only_ninf = mr == -(A)INFINITY;  // every value so far is -inf
   s = only_ninf ? ((n > 0) ? -fabs(s) : s) : t_sum;
   m = mr;
}

template < typename A >
__device__ __forceinline__ void lse_push(A& m, A& s, A v, A k)
{
   const A one[1] = {v};
   lse_fold< A, 1 >(m, s, one, 1, k);
}

// Two float columns per instruction: sm_100's packed f32x2 add / multiply /
// fma round each half like the scalar instruction, so the pair forms below
// give the scalar folds' results bit for bit in half the issue slots (the
// stream kernel is issue-bound when a lane holds two columns of a row).
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
// a - b as fma(b, -1, a): the exact difference, rounded once, like a subtraction.
__device__ __forceinline__ float2 sub2(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.f, -1.f), a); }

// lse_fold< float, N > on two columns at once (m, s, v[i] hold one value of
// each column): the maxima and exponentials per column, the differences,
// scalings, the sum tree and the rescale as packed pairs. The running state
// starts at (-FLT_MAX, 0) rather than (-inf, 0): a floor below every finite
// value, so -inf values add exp(-inf) = 0 and the state stays (-FLT_MAX, 0)
// while nothing else was seen, without the selects lse_fold spends on that
// case per fold (a value of -FLT_MAX itself adds exp(0) = 1). lse_floor_fix
// turns a state still at the floor back into lse_fold's encoding of it once
// the number of values folded is known.
constexpr float kLseFloor = -3.40282346638528859812e+38f;
template < int N >
__device__ __forceinline__ void lse_fold2(float2& m, float2& s, const float2 (&v)[N], int n, float k)
{
   const float ninf = -INFINITY;
   float2 t[N];
#pragma unroll
   for(int i = 0; i < N; ++i) t[i] = (i < n) ? v[i] : make_float2(ninf, ninf);
#pragma unroll
   for(int w = 1; w < N; w <<= 1)
#pragma unroll
      for(int i = 0; i + w < N; i += 2 * w) t[i] = make_float2(nanmax(t[i].x, t[i + w].x), nanmax(t[i].y, t[i + w].y));
   const float2 mr = make_float2(nanmax(m.x, t[0].x), nanmax(m.y, t[0].y));
   const float2 k2 = make_float2(k, k);
   float2 e[N];
#pragma unroll
   for(int i = 0; i < N; ++i) {
      if(i < n) {
         const float2 d = mul2(sub2(v[i], mr), k2);
         e[i] = make_float2(exp2_fast(d.x), exp2_fast(d.y));
      } else {
         e[i] = make_float2(0.f, 0.f);
      }
   }
#pragma unroll
   for(int w = 1; w < N; w <<= 1)
#pragma unroll
      for(int i = 0; i + w < N; i += 2 * w) e[i] = add2(e[i], e[i + w]);
   // (floor - mr) * k is -inf or a large negative number once mr is finite,
   // and exp2 of it 0; s is 0 there anyway
   const float2 d = mul2(sub2(m, mr), k2);
   s = fma2(s, make_float2(exp2_fast(d.x), exp2_fast(d.y)), e[0]);
   m = mr;
}

// Two 2-byte values packed in a 32-bit word (element 0 in the low half):
// their NaN-propagating maximum as a packed pair, the pair as floats, and the
// pair of -inf.
template < typename T >
__device__ __forceinline__ uint32_t max2_nan(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t max2_nan< __nv_bfloat16 >(uint32_t a, uint32_t b)
{
   uint32_t r;
   asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
   return r;
}
template <>
__device__ __forceinline__ uint32_t max2_nan< __half >(uint32_t a, uint32_t b)
{
   uint32_t r;
   asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
   return r;
}
template < typename T >
__device__ __forceinline__ float2 unpack2(uint32_t w);
template <>
__device__ __forceinline__ float2 unpack2< __nv_bfloat16 >(uint32_t w)
{
   return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack2< __half >(uint32_t w)
{
   __half2 h;
   memcpy(&h, &w, 4);
   return __half22float2(h);
}
template < typename T >
constexpr uint32_t kNegInf2 = sizeof(T) == 2 && std::is_same< T, __half >::value ? 0xfc00fc00u : 0xff80ff80u;

// lse_fold2 for 2-byte inputs held as packed pairs (w[i] = one word per edge):
// the maximum of the N new values per column is taken on the packed pairs
// (exact: a maximum of 2-byte values is one of them), and each exponent
// 2^((v - mr) k) is one fma, 2^(v k - mr k), with -mr k clamped to FLT_MAX so
// that a column still at the floor gives 2^-inf = 0 instead of inf - inf.
// The fma form rounds once instead of twice: its error, an ulp of mr k in the
// exponent, is far below the 2-byte output's rounding.
template < typename T, int N >
__device__ __forceinline__ void lse_fold2_packed(float2& m, float2& s, const uint32_t (&w)[N], int n, float k)
{
   uint32_t t = w[0];
#pragma unroll
   for(int i = 1; i < N; ++i)
      if(i < n) t = max2_nan< T >(t, w[i]);
   const float2 tf = unpack2< T >(t);
   const float2 mr = make_float2(nanmax(m.x, tf.x), nanmax(m.y, tf.y));
   const float2 k2 = make_float2(k, k);
   float2 nmk = mul2(mr, make_float2(-k, -k));
   nmk = make_float2(fminf(nmk.x, 3.402823466e38f), fminf(nmk.y, 3.402823466e38f));
   float2 e[N];
#pragma unroll
   for(int i = 0; i < N; ++i) {
      if(i < n) {
         const float2 d = fma2(unpack2< T >(w[i]), k2, nmk);
         e[i] = make_float2(exp2_fast(d.x), exp2_fast(d.y));
      } else {
         e[i] = make_float2(0.f, 0.f);
      }
   }
#pragma unroll
   for(int g = 1; g < N; g <<= 1)
#pragma unroll
      for(int i = 0; i + g < N; i += 2 * g) e[i] = add2(e[i], e[i + g]);
   const float2 d = fma2(m, k2, nmk);
   s = fma2(s, make_float2(exp2_fast(d.x), exp2_fast(d.y)), e[0]);
   m = mr;
}

// A state of lse_fold2 after `count` values, in lse_fold's encoding: still at
// the floor means no value (+0) or only -inf values (-0) with m = -inf.
__device__ __forceinline__ void lse_floor_fix(float& m, float& s, int count)
{
   if(m == kLseFloor && s == 0.f) {
      m = -INFINITY;
      s = count > 0 ? -0.f : 0.f;
   }
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
   const int32_t* has_dups;  // device flags of the plan: [0] some row holds more than one edge,
                             // [1] some row holds more than kShortRowEdges edges
   int short_rows;           // k_seg_rows_packed was launched too: the merge-path kernels and
                             // fixups leave plans without long rows to it
   int launch;               // host only: kernel families to launch (kLaunch*), all of them
                             // unless the host knows the plan's flags
   // kSumEpi epilogue (indexed sum / mean of the LGAN ops): the final value
   // of row R is epi_base[R] + sum / max(d, 1) with d = epi_div[R] when
   // epi_div is set, else the row's edge count when epi_count, else 1. The
   // dividing scatter (k_scatter_rows*<DIV>) divides plan row R by
   // max(epi_div[R], 1).
   const void* epi_base;
   const int64_t* epi_div;
   int epi_count;
   // logsumexp form (LseForm; the host sets the plain one unless asked for the
   // smoothed one): exponent scale, epsilon, 1 / beta, value of empty rows
   double lse_k;
   double lse_eps;
   double lse_inv_beta;
   double lse_empty;
};

template < typename A >
__device__ __forceinline__ LseForm< A > lse_form(const SegParams& p)
{
   return LseForm< A >{(A)p.lse_k, (A)p.lse_eps, (A)p.lse_inv_beta, (A)p.lse_empty};
}

// The merge-path kernels (and their fixups) serve the plan: some row holds
// more than one edge, and some row is long or k_seg_rows_packed was not launched.
__device__ __forceinline__ bool merge_path_runs(const SegParams& p)
{
   return p.has_dups[0] != 0 && (!p.short_rows || p.has_dups[1] != 0);
}

// Divisor of output row R in the SUM epilogue (at least 1; integers convert
// to the accumulator type before the clamp, as `counts.to(dtype).clamp_min(1)`).
template < typename T >
__device__ __forceinline__ typename AccOf< T >::type epi_divisor(const SegParams& p, int64_t R)
{
   using A = typename AccOf< T >::type;
   int64_t d = 1;
   if(p.epi_div)
      d = p.epi_div[R];
   else if(p.epi_count)
      d = (int64_t)p.row_ptr[R + 1] - (int64_t)p.row_ptr[R];
   const A a = (A)d;
   return a > A(1) ? a : A(1);
}

// v[k] <- base[R, col + k] + v[k] / divisor(R), k < N (an IEEE division, like
// the reference's `out / counts`; exact for a divisor of 1).
template < typename T, int N >
__device__ __forceinline__ void epi_apply(const SegParams& p, int64_t R, int64_t col,
                                          typename AccOf< T >::type (&v)[N])
{
   using A = typename AccOf< T >::type;
   const A d = epi_divisor< T >(p, R);
   const T* base = static_cast< const T* >(p.epi_base);
#pragma unroll
   for(int k = 0; k < N; ++k) {
      A r = v[k] / d;
      if(base) r += to_acc(base[R * p.emb + col + k]);
      v[k] = r;
   }
}

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

// 32-bit registers one lane spends on one gathered value (VB bytes per chunk,
// CH chunks, held in the accumulator type).
template < typename T, int VB, int CH >
__host__ __device__ constexpr int value_regs()
{
   return (VB / (int)sizeof(T)) * CH * (int)(sizeof(typename AccOf< T >::type) / 4);
}

// Loads in flight per lane group: about 16 registers of values (8 with the
// three loads per edge of the logsumexp backward).
template < typename T, int VB, int CH, int MODE >
__host__ __device__ constexpr int unroll_for()
{
   constexpr int budget = (MODE == kLseBwd) ? 8 : 16;
   constexpr int u = budget / value_regs< T, VB, CH >();
   return u < 1 ? 1 : (u > 8 ? 8 : u);
}

// Gathered row of output row g * 32 + lane: its last (or first) edge's gidx,
// -1 for rows without edges or past the end.
template < bool LAST >
__device__ __forceinline__ int32_t row_source(const SegParams& p, int64_t g, int64_t groups, int lane)
{
   const int64_t r = g * 32 + lane;
   int32_t src = -1;
   if(g < groups && r < p.num_rows) {
      const int32_t e0 = p.row_ptr[r];
      const int32_t e1 = p.row_ptr[r + 1];
      if(e1 > e0) src = p.gidx[LAST ? e1 - 1 : e0];
   }
   return src;
}

// Row map: one gathered row per output row.
//   kCopyLast: out[r] = table[gidx[last edge of r]], 0 without edges (fanout
//              forward; repeated slots keep the highest edge, as the reference
//              CPU loop leaves them).
//   kSum / kLse / kLseBwd: the same reductions as k_seg_reduce for plans whose
//              rows hold at most one edge (the kernel returns at once when the
//              plan's has_dups flag is set; k_seg_reduce runs instead).
// A warp owns groups of 32 consecutive rows: the lanes fetch the group's
// row_ptr / gidx entries with coalesced loads, prefetched one group ahead, then
// the whole warp moves one row per load with U rows in flight.
template < typename T, int VB, int CH, int MODE >
__global__ void __launch_bounds__(kThreads) k_row_map(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = VB / (int)sizeof(T);
   constexpr int U = unroll_for< T, VB, CH, (MODE == kLseBwd) ? kLseBwd : kSum >();
   if(MODE != kCopyLast && *p.has_dups) return;
   const int lane = threadIdx.x & 31;
   const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
   const T* table = static_cast< const T* >(p.table);
   const T* table2 = static_cast< const T* >(p.table2);
   const T* own = static_cast< const T* >(p.own);
   T* out = static_cast< T* >(p.out);
   const int64_t groups = (p.num_rows + 31) / 32;
   const A ninf = -(A)INFINITY;
   const LseForm< A > LF = lse_form< A >(p);

   int64_t g = warp;
   int32_t src_cur = row_source< MODE == kCopyLast >(p, g, groups, lane);
   for(; g < groups; g += nwarps) {
      const int32_t src_next = row_source< MODE == kCopyLast >(p, g + nwarps, groups, lane);
      const int64_t r0 = g * 32;
      const int nrows = (int)((p.num_rows - r0) < 32 ? (p.num_rows - r0) : 32);
      for(int cb = 0; cb < p.col_blocks; ++cb) {
         const Cols< CH > cols(p, cb, lane, VN);
         for(int base = 0; base < nrows; base += U) {
            A v[U][CH][VN];
            A w[(MODE == kLseBwd) ? U : 1][CH][VN];
            A o[(MODE == kLseBwd) ? U : 1][CH][VN];
            int32_t src[U];
#pragma unroll
            for(int u = 0; u < U; ++u) {
               src[u] = __shfl_sync(0xffffffffu, src_cur, (base + u) & 31);
               const bool live = base + u < nrows && src[u] >= 0;
#pragma unroll
               for(int c = 0; c < CH; ++c) {
                  if(live && cols.ok[c]) {
                     load_vec< T, VB >(table + (int64_t)src[u] * p.emb + cols.col[c], v[u][c]);
                     if(MODE == kLseBwd) {
                        const int ui = (MODE == kLseBwd) ? u : 0;
                        load_vec< T, VB >(table2 + (int64_t)src[u] * p.emb + cols.col[c], w[ui][c]);
                        load_vec< T, VB >(own + (r0 + base + u) * p.emb + cols.col[c], o[ui][c]);
                     }
                  }
               }
            }
#pragma unroll
            for(int u = 0; u < U; ++u) {
#pragma unroll
               for(int c = 0; c < CH; ++c) {
                  if(base + u >= nrows || !cols.ok[c]) continue;
                  A res[VN];
#pragma unroll
                  for(int k = 0; k < VN; ++k) {
                     if(src[u] < 0) {
                        res[k] = (MODE == kLse) ? LF.empty : A(0);
                     } else if(MODE == kCopyLast) {
                        res[k] = v[u][c][k];
                     } else if(sum_mode(MODE)) {
                        res[k] = A(0) + v[u][c][k];
                     } else if(MODE == kLse) {
                        A m = ninf, sacc = A(0);
                        lse_push(m, sacc, v[u][c][k], LF.k);
                        res[k] = lse_value(m, sacc, LF);
                     } else {
                        const int ui = (MODE == kLseBwd) ? u : 0;
                        res[k] = A(0) + v[u][c][k] * exp_k(o[ui][c][k] - w[ui][c][k], LF.k);
                     }
                  }
                  if(MODE == kSumEpi) epi_apply< T, VN >(p, r0 + base + u, cols.col[c], res);
                  store_vec< T, VB >(out + (r0 + base + u) * p.emb + cols.col[c], res);
               }
            }
         }
      }
      src_cur = src_next;
   }
}

// Packed shapes: rows of 16 to 256 bytes, a power of two times 16, with
// 16-byte aligned tables. L = row bytes / 16 lanes cover a row with 16-byte
// vectors and the warp's 32 / L lane groups work on different rows, so every
// load and store instruction moves 512 bytes whatever the row width (the
// narrow-vector shapes above move one row, 128 bytes for a 32-float or
// 64-bf16 row). Launchers select them with chmax == kPackedCh.
constexpr int kPackedCh = 0;

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast< const uint4* >(p)); }

// The elements of a 16-byte vector divided by d (rounded back to T).
template < typename T >
__device__ __forceinline__ uint4 div_raw16(uint4 v, typename AccOf< T >::type d)
{
   constexpr int VN = 16 / (int)sizeof(T);
   const T* e = reinterpret_cast< const T* >(&v);
   uint4 r;
   T* o = reinterpret_cast< T* >(&r);
#pragma unroll
   for(int k = 0; k < VN; ++k) o[k] = from_acc< T >(to_acc(e[k]) / d);
   return r;
}

// Row map with packed rows; same results as k_row_map.
template < typename T, int MODE >
__global__ void __launch_bounds__(kThreads, ((MODE == kLseBwd && sizeof(T) > 2) || MODE == kLse) ? 3 : 4)
   k_row_map_packed(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = 16 / (int)sizeof(T);
   // Row loads in flight per lane group (x3 for kLseBwd). Occupancy pays more
   // than deeper unrolling here (measured): 2-byte types hold 8 values per
   // vector, so their logsumexp backward keeps one row set in flight.
   constexpr int U = (MODE == kLseBwd && sizeof(T) == 2) ? 1 : 2;
   constexpr int UL = (MODE == kLseBwd) ? U : 1;
   if(MODE != kCopyLast && *p.has_dups) return;
   const int lane = threadIdx.x & 31;
   const int L = p.lanes;
   const int RPI = 32 / L;  // rows per load instruction
   const int sub = lane / L;
   const int64_t col = (int64_t)(lane - sub * L) * VN;
   const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
   const T* table = static_cast< const T* >(p.table);
   const T* table2 = static_cast< const T* >(p.table2);
   const T* own = static_cast< const T* >(p.own);
   T* out = static_cast< T* >(p.out);
   const int64_t groups = (p.num_rows + 31) / 32;
   const A ninf = -(A)INFINITY;
   const LseForm< A > LF = lse_form< A >(p);

   int64_t g = warp;
   int32_t src_cur = row_source< MODE == kCopyLast >(p, g, groups, lane);
   for(; g < groups; g += nwarps) {
      const int32_t src_next = row_source< MODE == kCopyLast >(p, g + nwarps, groups, lane);
      const int64_t r0 = g * 32;
      const int nrows = (int)((p.num_rows - r0) < 32 ? (p.num_rows - r0) : 32);
      for(int base = 0; base < nrows; base += RPI * U) {
         uint4 v[U], w[UL], o[UL];
         // kSumEpi: base rows and divisors, loaded with the table rows (rows of
         // this kernel hold at most one edge, so a count divisor is 1)
         constexpr int UE = (MODE == kSumEpi) ? U : 1;
         uint4 eb[UE];
         A ed[UE];
         int32_t src[U];
#pragma unroll
         for(int u = 0; u < U; ++u) {
            const int row = base + u * RPI + sub;
            src[u] = __shfl_sync(0xffffffffu, src_cur, row & 31);
            if(MODE == kSumEpi) {
               eb[u % UE] = make_uint4(0u, 0u, 0u, 0u);
               ed[u % UE] = A(1);
               if(row < nrows) {
                  if(p.epi_base) eb[u % UE] = ldg16(static_cast< const T* >(p.epi_base) + (r0 + row) * p.emb + col);
                  if(p.epi_div) {
                     const A dv = (A)p.epi_div[r0 + row];
                     ed[u % UE] = dv > A(1) ? dv : A(1);
                  }
               }
            }
            v[u] = make_uint4(0u, 0u, 0u, 0u);
            if(MODE == kLseBwd) {
               w[u % UL] = make_uint4(0u, 0u, 0u, 0u);
               o[u % UL] = make_uint4(0u, 0u, 0u, 0u);
            }
            if(row < nrows && src[u] >= 0) {
               v[u] = ldg16(table + (int64_t)src[u] * p.emb + col);
               if(MODE == kLseBwd) {
                  w[u % UL] = ldg16(table2 + (int64_t)src[u] * p.emb + col);
                  o[u % UL] = ldg16(own + (r0 + row) * p.emb + col);
               }
            }
         }
#pragma unroll
         for(int u = 0; u < U; ++u) {
            const int row = base + u * RPI + sub;
            if(row >= nrows) continue;
            const T* ev = reinterpret_cast< const T* >(&v[u]);
            const T* ew = reinterpret_cast< const T* >(&w[u % UL]);
            const T* eo = reinterpret_cast< const T* >(&o[u % UL]);
            uint4 r;
            T* er = reinterpret_cast< T* >(&r);
            A res[VN];
#pragma unroll
            for(int k = 0; k < VN; ++k) {
               if(src[u] < 0) {
                  res[k] = (MODE == kLse) ? LF.empty : A(0);
               } else if(MODE == kCopyLast) {
                  res[k] = to_acc(ev[k]);
               } else if(sum_mode(MODE)) {
                  res[k] = A(0) + to_acc(ev[k]);
               } else if(MODE == kLse) {
                  A m = ninf, sacc = A(0);
                  lse_push(m, sacc, to_acc(ev[k]), LF.k);
                  res[k] = lse_value(m, sacc, LF);
               } else {
                  res[k] = A(0) + to_acc(ev[k]) * exp_k(to_acc(eo[k]) - to_acc(ew[k]), LF.k);
               }
            }
            if(MODE == kSumEpi) {
               const T* ebk = reinterpret_cast< const T* >(&eb[u % UE]);
#pragma unroll
               for(int k = 0; k < VN; ++k) {
                  const A q = res[k] / ed[u % UE];
                  res[k] = p.epi_base ? q + to_acc(ebk[k]) : q;
               }
            }
#pragma unroll
            for(int k = 0; k < VN; ++k) er[k] = from_acc< T >(res[k]);
            *reinterpret_cast< uint4* >(out + (r0 + row) * p.emb + col) = r;
         }
      }
      src_cur = src_next;
   }
}

// Segment reduction for plans whose rows hold at most kShortRowEdges edges
// (some more than one), packed rows: the L = row bytes / 16 lanes of a lane
// group own one output row at a time and fold its edges kSrU at a time, all
// their loads in flight together (and, for kSumEpi / kLseBwd, the row's base /
// own row with them). No partials: a row never spans lane groups. Same
// results as the merge-path kernels up to the order of the additions.
constexpr int kSrU = 4;

template < typename T, int MODE >
__global__ void __launch_bounds__(kThreads) k_seg_rows_packed(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = 16 / (int)sizeof(T);
   constexpr int NT = (MODE == kLseBwd) ? 2 : 1;
   if(!p.has_dups[0] || p.has_dups[1]) return;
   const int lane = threadIdx.x & 31;
   const int L = p.lanes;
   const int RPI = 32 / L;
   const int sub = lane / L;
   const int64_t col = (int64_t)(lane - sub * L) * VN;
   const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
   const T* table = static_cast< const T* >(p.table);
   const T* table2 = static_cast< const T* >(p.table2);
   const T* own = static_cast< const T* >(p.own);
   T* out = static_cast< T* >(p.out);
   const A ninf = -(A)INFINITY;
   const LseForm< A > LF = lse_form< A >(p);
   for(int64_t r = warp * RPI + sub; r < p.num_rows; r += nwarps * RPI) {
      const int e0 = __ldg(p.row_ptr + r);
      const int e1 = __ldg(p.row_ptr + r + 1);
      uint4 side = make_uint4(0u, 0u, 0u, 0u);  // kSumEpi: base row; kLseBwd: own row
      A dv = A(1);
      if(MODE == kSumEpi) {
         if(p.epi_base) side = ldg16(static_cast< const T* >(p.epi_base) + r * p.emb + col);
         if(p.epi_div) {
            const A d = (A)__ldg(p.epi_div + r);
            dv = d > A(1) ? d : A(1);
         } else if(p.epi_count && e1 - e0 > 1) {
            dv = (A)(e1 - e0);
         }
      } else if(MODE == kLseBwd) {
         side = ldg16(own + r * p.emb + col);
      }
      A acc[VN], aux[VN];
#pragma unroll
      for(int k = 0; k < VN; ++k) {
         acc[k] = (MODE == kLse) ? ninf : A(0);
         aux[k] = A(0);
      }
      for(int j = e0; j < e1; j += kSrU) {
         const int n = (e1 - j) < kSrU ? (e1 - j) : kSrU;
         uint4 v[kSrU], w[NT == 2 ? kSrU : 1];
#pragma unroll
         for(int i = 0; i < kSrU; ++i) {
            v[i] = make_uint4(0u, 0u, 0u, 0u);
            if(NT == 2) w[i % (NT == 2 ? kSrU : 1)] = make_uint4(0u, 0u, 0u, 0u);
            if(i < n) {
               const int64_t g = __ldg(p.gidx + j + i);
               v[i] = ldg16(table + g * p.emb + col);
               if(NT == 2) w[i % (NT == 2 ? kSrU : 1)] = ldg16(table2 + g * p.emb + col);
            }
         }
#pragma unroll
         for(int k = 0; k < VN; ++k) {
            A x[kSrU];
#pragma unroll
            for(int i = 0; i < kSrU; ++i) x[i] = to_acc(reinterpret_cast< const T* >(&v[i])[k]);
            if(sum_mode(MODE)) {
#pragma unroll
               for(int i = 0; i < kSrU; ++i)
                  if(i < n) acc[k] += x[i];
            } else if(MODE == kLse) {
               lse_fold< A, kSrU >(acc[k], aux[k], x, n, LF.k);
            } else {
               const A o = to_acc(reinterpret_cast< const T* >(&side)[k]);
#pragma unroll
               for(int i = 0; i < kSrU; ++i)
                  if(i < n)
                     acc[k] += x[i] * exp_k(o - to_acc(reinterpret_cast< const T* >(&w[i % (NT == 2 ? kSrU : 1)])[k]), LF.k);
            }
         }
      }
      uint4 res;
      T* er = reinterpret_cast< T* >(&res);
#pragma unroll
      for(int k = 0; k < VN; ++k) {
         A f = (MODE == kLse) ? lse_value(acc[k], aux[k], LF) : acc[k];
         if(MODE == kSumEpi) {
            if(dv != A(1)) f = f / dv;
            if(p.epi_base) f += to_acc(reinterpret_cast< const T* >(&side)[k]);
         }
         er[k] = from_acc< T >(f);
      }
      *reinterpret_cast< uint4* >(out + r * p.emb + col) = res;
   }
}

// Scatter in plan-row order (fanout forward through the source plan): the
// warp walks its merge-path tile, loads each plan row's table row once (the
// next row's load is issued before the current row's stores) and stores it to
// out[gidx[j]] for every edge j of the row in the tile. No reduction, so rows
// that span tiles need no partials: each tile reloads the row it starts with.
template < typename T, int VB, int CH, bool DIV >
__global__ void __launch_bounds__(kThreads) k_scatter_rows(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = VB / (int)sizeof(T);
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
   if(j_begin == j_end) return;
   const T* table = static_cast< const T* >(p.table);
   T* out = static_cast< T* >(p.out);
   for(int cb = 0; cb < p.col_blocks; ++cb) {
      const Cols< CH > cols(p, cb, lane, VN);
      int gbase = j_begin, gcount = 0;
      int rbase = r_begin, rcount = 0;
      auto row_end = [&](int R) __attribute__((always_inline)) -> int {
         if(R >= r_end) return j_end;
         if(R - rbase >= rcount) {
            __syncwarp();
            rbase = R;
            rcount = (r_end - R) < kStage ? (r_end - R) : kStage;
            for(int i = lane; i < rcount; i += 32) sr[i] = p.row_ptr[R + 1 + i];
            __syncwarp();
         }
         const int e = sr[R - rbase];
         return e < j_end ? e : j_end;
      };
      auto load_row = [&](int R, A (&v)[CH][VN]) __attribute__((always_inline)) {
#pragma unroll
         for(int c = 0; c < CH; ++c)
            if(cols.ok[c]) load_vec< T, VB >(table + (int64_t)R * p.emb + cols.col[c], v[c]);
      };
      // DIV: rows are divided when they become current (after their loads
      // overlapped the previous row's stores).
      auto divide_row = [&](int R, A (&v)[CH][VN]) __attribute__((always_inline)) {
         if(DIV) {
            const A d = epi_divisor< T >(p, R);
#pragma unroll
            for(int c = 0; c < CH; ++c)
#pragma unroll
               for(int k = 0; k < VN; ++k) v[c][k] = v[c][k] / d;
         }
      };
      int R = r_begin;
      int j = j_begin;
      int e_end = row_end(R);
      while(e_end <= j) {  // rows that end before the tile's first edge (empty here)
         ++R;
         e_end = row_end(R);
      }
      A cur[CH][VN];
      load_row(R, cur);
      divide_row(R, cur);
      while(j < j_end) {
         // next row with edges in this tile, and its data, before storing this one
         int Rn = R + 1;
         int e_next = (Rn <= r_end) ? row_end(Rn) : j_end;
         while(Rn <= r_end && e_next <= e_end) {
            ++Rn;
            e_next = (Rn <= r_end) ? row_end(Rn) : j_end;
         }
         A nxt[CH][VN];
         const bool has_next = e_end < j_end;
         if(has_next) load_row(Rn, nxt);
         for(; j < e_end; ++j) {
            if(j >= gbase + gcount) {
               __syncwarp();
               gbase = j;
               gcount = (j_end - j) < kStage ? (j_end - j) : kStage;
               for(int i = lane; i < gcount; i += 32) sg[i] = p.gidx[j + i];
               __syncwarp();
            }
            const int64_t dst = sg[j - gbase];
#pragma unroll
            for(int c = 0; c < CH; ++c)
               if(cols.ok[c]) store_vec< T, VB >(out + dst * p.emb + cols.col[c], cur[c]);
         }
         if(!has_next) break;
#pragma unroll
         for(int c = 0; c < CH; ++c)
#pragma unroll
            for(int k = 0; k < VN; ++k) cur[c][k] = nxt[c][k];
         divide_row(Rn, cur);
         R = Rn;
         e_end = e_next;
      }
      __syncwarp();
   }
}

// k_scatter_rows with packed rows: the lane groups store the current row to
// 32 / L destinations per instruction.
template < typename T, bool DIV >
__global__ void __launch_bounds__(kThreads) k_scatter_rows_packed(SegParams p)
{
   constexpr int VN = 16 / (int)sizeof(T);
   __shared__ int32_t s_gidx[kWarps][kStage];
   __shared__ int32_t s_rend[kWarps][kStage];
   const int wib = threadIdx.x >> 5;
   const int64_t tile = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   if(tile >= p.num_tiles) return;
   const int lane = threadIdx.x & 31;
   const int L = p.lanes;
   const int RPI = 32 / L;  // destinations per store instruction
   const int sub = lane / L;
   const int64_t col = (int64_t)(lane - sub * L) * VN;
   int32_t* sg = s_gidx[wib];
   int32_t* sr = s_rend[wib];
   const int r_begin = p.tile_row[tile];
   const int j_begin = p.tile_edge[tile];
   const int r_end = p.tile_row[tile + 1];
   const int j_end = p.tile_edge[tile + 1];
   if(j_begin == j_end) return;
   const T* table = static_cast< const T* >(p.table);
   T* out = static_cast< T* >(p.out);
   int gbase = j_begin, gcount = 0;
   int rbase = r_begin, rcount = 0;
   auto row_end = [&](int R) __attribute__((always_inline)) -> int {
      if(R >= r_end) return j_end;
      if(R - rbase >= rcount) {
         __syncwarp();
         rbase = R;
         rcount = (r_end - R) < kStage ? (r_end - R) : kStage;
         for(int i = lane; i < rcount; i += 32) sr[i] = p.row_ptr[R + 1 + i];
         __syncwarp();
      }
      const int e = sr[R - rbase];
      return e < j_end ? e : j_end;
   };
   int R = r_begin;
   int j = j_begin;
   int e_end = row_end(R);
   while(e_end <= j) {  // rows that end before the tile's first edge (empty here)
      ++R;
      e_end = row_end(R);
   }
   // DIV: the next row and its divisor are loaded ahead and divided when the
   // row becomes current, so the loads overlap the current row's stores.
   using A = typename AccOf< T >::type;
   uint4 cur = ldg16(table + (int64_t)R * p.emb + col);
   if(DIV) cur = div_raw16< T >(cur, epi_divisor< T >(p, R));
   while(j < j_end) {
      int Rn = R + 1;
      int e_next = (Rn <= r_end) ? row_end(Rn) : j_end;
      while(Rn <= r_end && e_next <= e_end) {
         ++Rn;
         e_next = (Rn <= r_end) ? row_end(Rn) : j_end;
      }
      const bool has_next = e_end < j_end;
      uint4 nxt = cur;
      A dn = A(1);
      if(has_next) {
         nxt = ldg16(table + (int64_t)Rn * p.emb + col);
         if(DIV) dn = epi_divisor< T >(p, Rn);
      }
      for(; j < e_end; j += RPI) {
         const int need = (j + RPI) < e_end ? (j + RPI) : e_end;
         if(need > gbase + gcount) {
            __syncwarp();
            gbase = j;
            gcount = (j_end - j) < kStage ? (j_end - j) : kStage;
            for(int i = lane; i < gcount; i += 32) sg[i] = p.gidx[j + i];
            __syncwarp();
         }
         const int jj = j + sub;
         if(jj < e_end) *reinterpret_cast< uint4* >(out + (int64_t)sg[jj - gbase] * p.emb + col) = cur;
      }
      j = e_end;
      if(!has_next) break;
      cur = DIV ? div_raw16< T >(nxt, dn) : nxt;
      R = Rn;
      e_end = e_next;
   }
   __syncwarp();
}

// Logsumexp backward in destination order, for message rows used at most
// once (packed rows): walks the forward's plan (rows = destination rows,
// gidx = message rows); each destination row's grad_out and lse rows are read
// once, and every message row m of it gets
// grad_rel[m] = grad_out[d] * exp(rel[m] - lse[d]) (the row-map expression,
// bit for bit). Two store groups of 32 / L message rows are loaded per step.
template < typename T >
__global__ void __launch_bounds__(kThreads) k_scatter_lse_bwd_packed(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = 16 / (int)sizeof(T);
   __shared__ int32_t s_gidx[kWarps][kStage];
   __shared__ int32_t s_rend[kWarps][kStage];
   const int wib = threadIdx.x >> 5;
   const int64_t tile = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   if(tile >= p.num_tiles) return;
   const int lane = threadIdx.x & 31;
   const int L = p.lanes;
   const int RPI = 32 / L;
   const int sub = lane / L;
   const int64_t col = (int64_t)(lane - sub * L) * VN;
   int32_t* sg = s_gidx[wib];
   int32_t* sr = s_rend[wib];
   const int r_begin = p.tile_row[tile];
   const int j_begin = p.tile_edge[tile];
   const int r_end = p.tile_row[tile + 1];
   const int j_end = p.tile_edge[tile + 1];
   if(j_begin == j_end) return;
   const T* gout = static_cast< const T* >(p.table);   // grad_out, by destination row
   const T* lse = static_cast< const T* >(p.table2);   // forward output, by destination row
   const T* rel = static_cast< const T* >(p.own);      // messages, by message row
   T* out = static_cast< T* >(p.out);                  // grad_rel, by message row
   const A lse_k = (A)p.lse_k;
   int gbase = j_begin, gcount = 0;
   int rbase = r_begin, rcount = 0;
   auto row_end = [&](int R) __attribute__((always_inline)) -> int {
      if(R >= r_end) return j_end;
      if(R - rbase >= rcount) {
         __syncwarp();
         rbase = R;
         rcount = (r_end - R) < kStage ? (r_end - R) : kStage;
         for(int i = lane; i < rcount; i += 32) sr[i] = p.row_ptr[R + 1 + i];
         __syncwarp();
      }
      const int e = sr[R - rbase];
      return e < j_end ? e : j_end;
   };
   int R = r_begin;
   int j = j_begin;
   int e_end = row_end(R);
   while(e_end <= j) {
      ++R;
      e_end = row_end(R);
   }
   uint4 cg = ldg16(gout + (int64_t)R * p.emb + col);
   uint4 co = ldg16(lse + (int64_t)R * p.emb + col);
   while(j < j_end) {
      int Rn = R + 1;
      int e_next = (Rn <= r_end) ? row_end(Rn) : j_end;
      while(Rn <= r_end && e_next <= e_end) {
         ++Rn;
         e_next = (Rn <= r_end) ? row_end(Rn) : j_end;
      }
      const bool has_next = e_end < j_end;
      uint4 ng = cg, no = co;
      if(has_next) {
         ng = ldg16(gout + (int64_t)Rn * p.emb + col);
         no = ldg16(lse + (int64_t)Rn * p.emb + col);
      }
      const T* eg = reinterpret_cast< const T* >(&cg);
      const T* eo = reinterpret_cast< const T* >(&co);
      for(; j < e_end; j += 2 * RPI) {
         const int need = (j + 2 * RPI) < e_end ? (j + 2 * RPI) : e_end;
         if(need > gbase + gcount) {
            __syncwarp();
            gbase = j;
            gcount = (j_end - j) < kStage ? (j_end - j) : kStage;
            for(int i = lane; i < gcount; i += 32) sg[i] = p.gidx[j + i];
            __syncwarp();
         }
         int64_t m[2];
         uint4 v[2];
#pragma unroll
         for(int h = 0; h < 2; ++h) {
            const int jj = j + h * RPI + sub;
            m[h] = jj < e_end ? (int64_t)sg[jj - gbase] : -1;
            v[h] = make_uint4(0u, 0u, 0u, 0u);
            if(m[h] >= 0) v[h] = ldg16(rel + m[h] * p.emb + col);
         }
#pragma unroll
         for(int h = 0; h < 2; ++h) {
            if(m[h] < 0) continue;
            const T* ev = reinterpret_cast< const T* >(&v[h]);
            uint4 r;
            T* er = reinterpret_cast< T* >(&r);
#pragma unroll
            for(int k = 0; k < VN; ++k)
               er[k] = from_acc< T >(A(0) + to_acc(eg[k]) * exp_k(to_acc(ev[k]) - to_acc(eo[k]), lse_k));
            *reinterpret_cast< uint4* >(out + m[h] * p.emb + col) = r;
         }
      }
      j = e_end;
      if(!has_next) break;
      cg = ng;
      co = no;
      R = Rn;
      e_end = e_next;
   }
   __syncwarp();
}

// Zero rows of `out` whose bit in the cover bitmap is clear.
template < typename T, int VB, int CH >
__global__ void __launch_bounds__(kThreads) k_zero_uncovered(SegParams p, const uint32_t* __restrict__ cover,
                                                             int64_t rows)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = VB / (int)sizeof(T);
   const int lane = threadIdx.x & 31;
   const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
   T* out = static_cast< T* >(p.out);
   A zero[VN];
#pragma unroll
   for(int k = 0; k < VN; ++k) zero[k] = A(0);
   for(int64_t base = warp * 32; base < rows; base += nwarps * 32) {
      const int64_t r = base + lane;
      const unsigned todo = __ballot_sync(0xffffffffu, r < rows && ((cover[base >> 5] >> lane) & 1u) == 0u);
      for(unsigned m = todo; m; m &= m - 1) {
         const int64_t row = base + __ffs(m) - 1;
         for(int cb = 0; cb < p.col_blocks; ++cb) {
            const Cols< CH > cols(p, cb, lane, VN);
#pragma unroll
            for(int c = 0; c < CH; ++c)
               if(cols.ok[c]) store_vec< T, VB >(out + row * p.emb + cols.col[c], zero);
         }
      }
   }
}

// Segment reduction over one merge-path tile per warp.
//
// A row is covered by `lanes` lanes (VB bytes each, 16 when possible), so the
// warp holds G = 32 / lanes lane groups and one load instruction moves G
// gathered rows. The tile's edges are consumed as one stream, G * U at a time
// whatever the row lengths: group g takes edges j + g, j + g + G, ... The warp
// first resolves the row of every edge of the batch from the staged row ends
// (shared memory, uniform walk), issues the loads, then folds the values into
// the per-group accumulators in edge order, finishing rows as the stream
// crosses their ends (a finished row folds its G group accumulators with
// shuffles). Rows that began in an earlier tile are written as a head partial,
// the row still open at the end of the tile as a tail partial; k_fixup
// combines them in tile order.
template < typename T, int VB, int CH, int MODE >
__global__ void __launch_bounds__(kThreads, (value_regs< T, VB, CH >() <= 4) ? 3 : 2) k_seg_reduce(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = VB / (int)sizeof(T);
   constexpr int U = unroll_for< T, VB, CH, MODE >();
   __shared__ int32_t s_gidx[kWarps][kStage];
   __shared__ int32_t s_rend[kWarps][kStage];
   const int wib = threadIdx.x >> 5;
   const int64_t tile = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
   if(tile >= p.num_tiles || !merge_path_runs(p)) return;
   const int lane = threadIdx.x & 31;
   const int L = p.lanes;
   const int G = 32 / L;
   const int grp = lane / L;
   const int sub = lane % L;
   const LseForm< A > LF = lse_form< A >(p);
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
      int64_t col[CH];
      bool ok[CH];
#pragma unroll
      for(int c = 0; c < CH; ++c) {
         col[c] = cb * p.block_cols + (int64_t)(c * L + sub) * VN;
         ok[c] = c < p.ch && col[c] < p.emb;
      }
      int gbase = j_begin, gcount = 0;
      int rbase = r_begin, rcount = 0;
      // End (exclusive edge index) of row R < r_end, from the staged row ends.
      auto row_end = [&](int R) __attribute__((always_inline)) -> int {
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
      auto reset = [&]() __attribute__((always_inline)) {
#pragma unroll
         for(int c = 0; c < CH; ++c)
#pragma unroll
            for(int k = 0; k < VN; ++k) {
               acc[c][k] = (MODE == kLse) ? ninf : A(0);
               aux[c][k] = A(0);
            }
      };
      // Folds the G group accumulators of the open row (every lane ends up
      // with the row's total).
      auto fold = [&]() __attribute__((always_inline)) {
         for(int off = L; off < 32; off <<= 1) {
#pragma unroll
            for(int c = 0; c < CH; ++c)
#pragma unroll
               for(int k = 0; k < VN; ++k) {
                  const A om = __shfl_xor_sync(0xffffffffu, acc[c][k], off);
                  if(MODE == kLse) {
                     const A os = __shfl_xor_sync(0xffffffffu, aux[c][k], off);
                     lse_merge(acc[c][k], aux[c][k], om, os, LF.k);
                  } else {
                     acc[c][k] += om;
                  }
               }
         }
      };
      // Finishes row R: final output, or the head partial when it began earlier.
      auto flush = [&](int R) __attribute__((always_inline)) {
         fold();
         const bool head = (R == r_begin) && began_before;
         if(grp == 0) {
#pragma unroll
            for(int c = 0; c < CH; ++c) {
               if(!ok[c]) continue;
               if(head) {
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
                     fin[k] = (MODE == kLse) ? lse_value(acc[c][k], aux[c][k], LF) : acc[c][k];
                  if(MODE == kSumEpi) epi_apply< T, VN >(p, R, col[c], fin);
                  store_vec< T, VB >(out + (int64_t)R * p.emb + col[c], fin);
               }
            }
         }
         if(head) head_row = R;
         reset();
      };
      auto fold_in = [&](const A (&val)[CH][VN], const A (&w2)[CH][VN], const A (&o2)[CH][VN]) {
#pragma unroll
         for(int c = 0; c < CH; ++c) {
            if(!ok[c]) continue;
#pragma unroll
            for(int k = 0; k < VN; ++k) {
               if(sum_mode(MODE))
                  acc[c][k] += val[c][k];
               else if(MODE == kLse)
                  lse_push(acc[c][k], aux[c][k], val[c][k], LF.k);
               else
                  acc[c][k] += val[c][k] * exp_k(o2[c][k] - w2[c][k], LF.k);
            }
         }
      };

      reset();
      int R = r_begin;   // open row (all rows before it are finished)
      int Rw = r_begin;  // walker: row of the next edge
      int rend_w = (Rw < r_end) ? row_end(Rw) : INT_MAX;
      bool pending = false;  // the open row holds edges of this tile
      const int step = G * U;
      for(int j = j_begin; j < j_end; j += step) {
         const int nb = (j_end - j) < step ? (j_end - j) : step;
         if(j + nb > gbase + gcount) {
            __syncwarp();
            gbase = j;
            gcount = (j_end - j) < kStage ? (j_end - j) : kStage;
            for(int i = lane; i < gcount; i += 32) sg[i] = p.gidx[j + i];
            __syncwarp();
         }
         // Row of this group's edges (rr) and of the last edge of each sub-batch (rl).
         int rr[U];
         int rl[U];
#pragma unroll
         for(int u = 0; u < U; ++u) {
            rr[u] = INT_MAX;
            rl[u] = Rw;
            for(int g = 0; g < G; ++g) {
               const int e = u * G + g;
               if(e < nb) {
                  while(rend_w <= j + e) {
                     ++Rw;
                     rend_w = (Rw < r_end) ? row_end(Rw) : INT_MAX;
                  }
                  if(g == grp) rr[u] = Rw;
                  rl[u] = Rw;
               }
            }
         }
         A v[U][CH][VN];
         A w[(MODE == kLseBwd) ? U : 1][CH][VN];
         A o[(MODE == kLseBwd) ? U : 1][CH][VN];
#pragma unroll
         for(int u = 0; u < U; ++u) {
            const int e = u * G + grp;
            const int32_t g = (e < nb) ? sg[j + e - gbase] : 0;
#pragma unroll
            for(int c = 0; c < CH; ++c) {
               if(e < nb && ok[c]) {
                  load_vec< T, VB >(table + (int64_t)g * p.emb + col[c], v[u][c]);
                  if(MODE == kLseBwd) {
                     const int ui = (MODE == kLseBwd) ? u : 0;
                     load_vec< T, VB >(table2 + (int64_t)g * p.emb + col[c], w[ui][c]);
                     load_vec< T, VB >(own + (int64_t)rr[u] * p.emb + col[c], o[ui][c]);
                  }
               }
            }
         }
#pragma unroll
         for(int u = 0; u < U; ++u) {
            if(u * G >= nb) continue;
            const int ui = (MODE == kLseBwd) ? u : 0;
            bool added = false;
            if(rr[u] == R) {
               fold_in(v[u], w[ui], o[ui]);
               added = true;
            }
            while(R < rl[u]) {
               flush(R);
               ++R;
               if(!added && rr[u] == R) {
                  fold_in(v[u], w[ui], o[ui]);
                  added = true;
               }
            }
            pending = true;
         }
      }
      while(R < r_end) {
         flush(R);
         pending = false;
         ++R;
      }
      if(pending) {
         fold();
         if(grp == 0) {
#pragma unroll
            for(int c = 0; c < CH; ++c) {
               if(!ok[c]) continue;
               const int64_t off = tile * p.emb + col[c];
#pragma unroll
               for(int k = 0; k < VN; ++k) {
                  tail_val[off + k] = acc[c][k];
                  if(MODE == kLse) tail_aux[off + k] = aux[c][k];
               }
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

// ---- shared-memory gather pipeline ---------------------------------------------

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem)
{
   const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
   asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
// Same, with the destination as a shared-window address.
__device__ __forceinline__ void cp_async16_s(unsigned s, const void* gmem)
{
   asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template < int N >
__device__ __forceinline__ void cp_async_wait()
{
   asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// PB bytes of T (PB in {2, 4, 8, 16, 32}) <-> accumulator values.
template < typename T, int PB >
__device__ __forceinline__ void load_chunk(const T* p, typename AccOf< T >::type (&out)[PB / sizeof(T)])
{
   constexpr int W = PB < 16 ? PB : 16;
   constexpr int per = W / (int)sizeof(T);
#pragma unroll
   for(int i = 0; i < PB / W; ++i) {
      using R = typename Raw< W >::type;
      const R r = *reinterpret_cast< const R* >(p + i * per);
      const T* e = reinterpret_cast< const T* >(&r);
#pragma unroll
      for(int k = 0; k < per; ++k) out[i * per + k] = to_acc(e[k]);
   }
}

template < typename T, int PB >
__device__ __forceinline__ void load_chunk_global(const T* p, typename AccOf< T >::type (&out)[PB / sizeof(T)])
{
   constexpr int W = PB < 16 ? PB : 16;
   constexpr int per = W / (int)sizeof(T);
#pragma unroll
   for(int i = 0; i < PB / W; ++i) {
      typename AccOf< T >::type part[per];
      load_vec< T, W >(p + i * per, part);
#pragma unroll
      for(int k = 0; k < per; ++k) out[i * per + k] = part[k];
   }
}

template < typename T, int PB >
__device__ __forceinline__ void store_chunk(T* p, const typename AccOf< T >::type (&in)[PB / sizeof(T)])
{
   constexpr int W = PB < 16 ? PB : 16;
   constexpr int per = W / (int)sizeof(T);
#pragma unroll
   for(int i = 0; i < PB / W; ++i) {
      typename AccOf< T >::type part[per];
#pragma unroll
      for(int k = 0; k < per; ++k) part[k] = in[i * per + k];
      store_vec< T, W >(p + i * per, part);
   }
}

// Tuning constants of the stream kernel (measured on B200; the values below
// are the defaults, builds may override them to measure alternatives).
#ifndef RELM_MP_STREAM_STAGE_BYTES
#define RELM_MP_STREAM_STAGE_BYTES 4096
#endif
#ifndef RELM_MP_STREAM_MIN_BLOCKS
#define RELM_MP_STREAM_MIN_BLOCKS 7
#endif
#ifndef RELM_MP_STREAM_STAGES
#define RELM_MP_STREAM_STAGES 2
#endif
constexpr int kStreamWarps = 4;
constexpr int kStreamThreads = kStreamWarps * 32;
constexpr int kStreamStages = RELM_MP_STREAM_STAGES;
constexpr int kStreamStageBytes = RELM_MP_STREAM_STAGE_BYTES;  // per warp, stage and gathered table
constexpr int kStreamMeta = 96;         // staged gidx / row-end entries per warp

// Per-warp shared memory: the stages, staged gidx and row ends, and for the
// SUM epilogue the staged divisors (8 bytes each).
__host__ __device__ constexpr int stream_warp_bytes(int tables, bool epi = false)
{
   return tables * kStreamStages * kStreamStageBytes + 2 * kStreamMeta * 4 + (epi ? kStreamMeta * 8 : 0);
}

// Prefetch of a contiguous range to L2 (16-byte aligned, a multiple of 16 bytes).
__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes)
{
   asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Segment reduction over one merge-path tile per warp, with the gathered rows
// brought into shared memory by cp.async ahead of use.
//
// A column block of CBW bytes of each gathered row (the whole row up to 1 KB)
// is split over `lanes` lanes of PB bytes. The tile's edges are fetched B rows
// per stage, kStreamStages - 1 stages ahead of the one being folded: the copies
// need no registers, so the bytes in flight per SM no longer depend on register
// pressure, and folding an edge costs one shared load and the arithmetic. The
// fold walks the edges in order, finishing rows as it crosses their ends; rows
// that began in an earlier tile go out as head partials, the row still open at
// the end as the tail partial (combined by k_fixup in tile order).
//
// FULL: rows of exactly 32 * PB bytes (one column block, all 32 lanes): the
// block width, rows per stage and the copy layout are compile-time constants,
// so a full batch issues its copies unrolled and every shared load of the
// fold takes an immediate offset.
template < typename T, int PB, int MODE, bool FULL >
__global__ void __launch_bounds__(kStreamThreads, RELM_MP_STREAM_MIN_BLOCKS) k_seg_stream(SegParams p)
{
   using A = typename AccOf< T >::type;
   constexpr int VN = PB / (int)sizeof(T);
   constexpr int NT = (MODE == kLseBwd) ? 2 : 1;
   // float accumulators, an even number of columns per lane: the folds work on column pairs
   constexpr bool kPairs = sizeof(A) == 4 && VN % 2 == 0;
   // logsumexp on column pairs: running states start at the floor (lse_fold2)
   constexpr bool kFloor = kPairs && MODE == kLse;
   // the flush counts each row's edges in the tile (rows without any are written
   // straight from the empty-row value: most rows of a Zipf fan-in are empty);
   // kSumEpi rows take their base row instead
   constexpr bool kCount = MODE != kSumEpi;
   static_assert(!FULL || PB <= 16, "FULL rows take at most 32 16-byte chunks");
   extern __shared__ __align__(16) unsigned char smem[];
   const int wib = threadIdx.x >> 5;
   const int lane = threadIdx.x & 31;
   const int64_t tile = (int64_t)blockIdx.x * kStreamWarps + wib;
   if(tile >= p.num_tiles || !merge_path_runs(p)) return;
   // kSumEpi with 8..16-byte lane chunks: divisors staged beside the row ends,
   // base rows prefetched to L2 per tile and into registers two rows ahead
   // (rows of 32-byte lane chunks keep the plain epilogue: their two extra
   // register rows would spill)
   constexpr bool PF = MODE == kSumEpi && PB <= 16;
   // (the divisor staging takes shared memory only when there is a divisor array)
   unsigned char* wbase = smem + (size_t)wib * stream_warp_bytes(NT, MODE == kSumEpi && p.epi_div);
   int32_t* sg = reinterpret_cast< int32_t* >(wbase + NT * kStreamStages * kStreamStageBytes);
   int32_t* sr = sg + kStreamMeta;
   A* sdv = reinterpret_cast< A* >(sr + kStreamMeta);  // kSumEpi: divisor of row rbase + i
   constexpr int kFullCBW = 32 * PB;
   constexpr int kFullB = (kStreamStageBytes / kFullCBW) < 32 ? (kStreamStageBytes / kFullCBW) : 32;
   const int CBW = FULL ? kFullCBW : (int)p.block_cols * (int)sizeof(T);  // bytes of a column block
   const int B = FULL ? kFullB : p.ch;                                     // rows per stage
   const bool lane_ok = FULL || lane < p.lanes;
   const int64_t row_bytes = FULL ? (int64_t)kFullCBW : p.emb * (int64_t)sizeof(T);
   const int ncb = FULL ? 1 : p.col_blocks;
   constexpr int kFullChunks = kFullCBW / 16;  // copies of 16 bytes per row
   constexpr int kFullCopies = kFullB / (kFullChunks <= 32 ? 32 / kFullChunks : 1);  // per lane and full batch
   const int r_begin = p.tile_row[tile];
   const int j_begin = p.tile_edge[tile];
   const int r_end = p.tile_row[tile + 1];
   const int j_end = p.tile_edge[tile + 1];
   const bool began_before = p.row_ptr[r_begin] < j_begin;
   const char* table = static_cast< const char* >(p.table);
   const char* table2 = static_cast< const char* >(p.table2);
   const T* own = static_cast< const T* >(p.own);
   T* out = static_cast< T* >(p.out);
   A* head_val = static_cast< A* >(p.head_val);
   A* tail_val = static_cast< A* >(p.tail_val);
   A* head_aux = static_cast< A* >(p.head_aux);
   A* tail_aux = static_cast< A* >(p.tail_aux);
   const A ninf = -(A)INFINITY;
   const LseForm< A > LF = lse_form< A >(p);
   const int nbatches = (j_end - j_begin + B - 1) / B;
   const int chunks = CBW / 16;
   int head_row = -1;
   int tail_row = -1;

   for(int cb = 0; cb < ncb; ++cb) {
      const int64_t cbyte = (int64_t)cb * CBW;
      const int64_t col = (cbyte + (int64_t)lane * PB) / (int64_t)sizeof(T);
      int gbase = j_begin, gcount = 0;
      int rbase = r_begin, rcount = 0;
      // The window after the staged one (gidx entries, row ends) is loaded into
      // registers when a window is staged: the next refill stores values that
      // arrived long before instead of waiting on global loads.
      constexpr int MQ = kStreamMeta / 32;
      int32_t g_next[MQ], r_next[MQ];
      int g_next_at = -1, r_next_at = -1;
      auto prefetch_g = [&](int j) __attribute__((always_inline)) {
         g_next_at = j;
#pragma unroll
         for(int q = 0; q < MQ; ++q) {
            const int i = j + lane + 32 * q;
            g_next[q] = i < j_end ? p.gidx[i] : 0;
         }
      };
      auto prefetch_r = [&](int R0) __attribute__((always_inline)) {
         r_next_at = R0;
#pragma unroll
         for(int q = 0; q < MQ; ++q) {
            const int R1 = R0 + lane + 32 * q;
            r_next[q] = R1 < r_end ? p.row_ptr[R1 + 1] : 0;
         }
      };
      auto row_end = [&](int R) __attribute__((always_inline)) -> int {
         if(R - rbase >= rcount) {
            __syncwarp();
            rbase = R;
            rcount = (r_end - R) < kStreamMeta ? (r_end - R) : kStreamMeta;
            if(R == r_next_at) {
#pragma unroll
               for(int q = 0; q < MQ; ++q)
                  if(lane + 32 * q < rcount) sr[lane + 32 * q] = r_next[q];
            } else {
               for(int i = lane; i < rcount; i += 32) sr[i] = p.row_ptr[R + 1 + i];
            }
            if(R + rcount < r_end) prefetch_r(R + rcount);
            for(int i = lane; i < rcount; i += 32) {
               if(PF && p.epi_div) {
                  const A dv = (A)p.epi_div[R + i];
                  sdv[i] = dv > A(1) ? dv : A(1);
               }
            }
            __syncwarp();
         }
         return sr[R - rbase];
      };
      // Copies batch k (rows j_begin + k*B ...) into stage k % kStreamStages.
      // Lane l copies 16-byte chunk (l mod chunks) of rows l / chunks, + 32 / chunks, ...
      // (chunks is a power of two; wider rows give a lane several chunks). With
      // chunks <= 32 a lane's copies of one batch are 512 bytes apart in shared
      // memory, and its source offsets are 32-bit row ids times the row size.
      const int cl = lane & (chunks - 1);
      const int b_first = chunks <= 32 ? lane / chunks : 0;
      const int rpi = chunks <= 32 ? 32 / chunks : 1;
      const unsigned s_lane = (unsigned)__cvta_generic_to_shared(wbase) + (unsigned)(b_first * CBW + cl * 16);
      const char* g_lane = table + cbyte + cl * 16;
      const char* g2_lane = (NT == 2) ? table2 + cbyte + cl * 16 : nullptr;
      const unsigned rbytes = (unsigned)row_bytes;
      auto issue = [&](int k) __attribute__((always_inline)) {
         if(k < nbatches) {
            const int j0 = j_begin + k * B;
            const int nb = (j_end - j0) < B ? (j_end - j0) : B;
            if(j0 + nb > gbase + gcount) {
               __syncwarp();
               gbase = j0;
               gcount = (j_end - j0) < kStreamMeta ? (j_end - j0) : kStreamMeta;
               if(j0 == g_next_at) {
#pragma unroll
                  for(int q = 0; q < MQ; ++q)
                     if(lane + 32 * q < gcount) sg[lane + 32 * q] = g_next[q];
               } else {
                  for(int i = lane; i < gcount; i += 32) sg[i] = p.gidx[j0 + i];
               }
               if(j0 + gcount < j_end) prefetch_g(j0 + gcount);
               __syncwarp();
            }
            unsigned char* st = wbase + (k % kStreamStages) * kStreamStageBytes;
            const int32_t* sgb = sg + (j0 - gbase);
            if(FULL && nb == B) {
               const unsigned sa = s_lane + (unsigned)((k % kStreamStages) * kStreamStageBytes);
#pragma unroll
               for(int i = 0; i < kFullCopies; ++i) {
                  const uint64_t off = (uint64_t)(unsigned)sgb[b_first + i * rpi] * rbytes;
                  cp_async16_s(sa + 512u * i, g_lane + off);
                  if(NT == 2) cp_async16_s(sa + 512u * i + (unsigned)(kStreamStages * kStreamStageBytes), g2_lane + off);
               }
            } else if(chunks <= 32) {
               unsigned sa = s_lane + (unsigned)((k % kStreamStages) * kStreamStageBytes);
               for(int b = b_first; b < nb; b += rpi, sa += 512u) {
                  const uint64_t off = (uint64_t)(unsigned)sgb[b] * rbytes;
                  cp_async16_s(sa, g_lane + off);
                  if(NT == 2) cp_async16_s(sa + (unsigned)(kStreamStages * kStreamStageBytes), g2_lane + off);
               }
            } else {
               for(int b = 0; b < nb; ++b) {
                  const int64_t roff = (int64_t)sgb[b] * row_bytes + cbyte;
                  for(int c = lane; c < chunks; c += 32) {
                     cp_async16(st + b * CBW + c * 16, table + roff + c * 16);
                     if(NT == 2)
                        cp_async16(st + kStreamStages * kStreamStageBytes + b * CBW + c * 16, table2 + roff + c * 16);
                  }
               }
            }
         }
         cp_async_commit();
      };
      A acc[VN];
      A aux[VN];
      A ownv[VN];
      // kSumEpi: the divisor is the staged row's edge count (row ends already
      // walked) or its staged divisor, and the base row is read at the flush
      // from L2 (the tile's base rows are prefetched there at its start). The
      // kernel is issue-bound on short rows, so the epilogue is kept to a few
      // instructions: no division when the divisor is 1.
      int e_rstart = 0;
      auto epi_finish = [&](int Rr, int cnt, A (&fin)[VN]) __attribute__((always_inline)) {
         if constexpr(PF) {
            const A d = p.epi_div ? sdv[Rr - rbase] : ((p.epi_count && cnt > 1) ? (A)cnt : A(1));
            if(d != A(1)) {
#pragma unroll
               for(int k_ = 0; k_ < VN; ++k_) fin[k_] = fin[k_] / d;
            }
            if(p.epi_base) {
               A b[VN];
               load_chunk_global< T, PB >(static_cast< const T* >(p.epi_base) + (int64_t)Rr * p.emb + col, b);
#pragma unroll
               for(int k_ = 0; k_ < VN; ++k_) fin[k_] += b[k_];
            }
         }
      };
      if(kCount) e_rstart = j_begin;  // the open row's first edge in this tile
      // value of a row without edges (the reduction of nothing)
      A empty_[VN];
#pragma unroll
      for(int k_ = 0; k_ < VN; ++k_) empty_[k_] = (MODE == kLse) ? LF.empty : A(0);
      if(PF) {
         if(cb == 0 && lane == 0 && p.epi_base) {  // this tile's base rows, to L2
            const int r_last = r_end < (int)p.num_rows ? r_end : (int)p.num_rows - 1;
            const char* b0 = static_cast< const char* >(p.epi_base) + (int64_t)r_begin * row_bytes;
            int64_t left = (int64_t)(r_last - r_begin + 1) * row_bytes;
            for(; left > 0; b0 += 32768, left -= 32768) prefetch_l2(b0, (unsigned)(left < 32768 ? left : 32768));
         }
         if(p.epi_count) e_rstart = p.row_ptr[r_begin];
      }
#define RELM_MP_STREAM_RESET()                                  \
   do {                                                         \
      _Pragma("unroll") for(int k_ = 0; k_ < VN; ++k_)          \
      {                                                         \
         acc[k_] = (MODE == kLse) ? (kFloor ? (A)kLseFloor : ninf) : A(0); \
         aux[k_] = A(0);                                        \
      }                                                         \
   } while(0)
      // Finishes row R_: final output, or the head partial when it began earlier.
#define RELM_MP_STREAM_FLUSH(R_, RE_)                                                            \
   do {                                                                                         \
      const bool head_ = ((R_) == r_begin) && began_before;                                     \
      int cnt_ = 0;                                                                             \
      if(PF || kCount) { /* RE_: row_end(R_), which also holds R_'s divisor (PF) */           \
         const int re_ = (RE_);                                                                 \
         cnt_ = re_ - e_rstart;                                                                 \
         e_rstart = re_;                                                                        \
      }                                                                                         \
      if(kCount && cnt_ == 0 && !head_) { /* no edge: the empty-row value, state untouched */  \
         if(lane_ok) store_chunk< T, PB >(out + (int64_t)(R_)*p.emb + col, empty_);             \
         break;                                                                                 \
      }                                                                                         \
      if constexpr(kFloor) {                                                                    \
         _Pragma("unroll") for(int k_ = 0; k_ < VN; ++k_) lse_floor_fix(acc[k_], aux[k_], cnt_); \
      }                                                                                         \
      if(lane_ok) {                                                                             \
         if(head_) {                                                                            \
            const int64_t off_ = tile * p.emb + col;                                            \
            _Pragma("unroll") for(int k_ = 0; k_ < VN; ++k_)                                    \
            {                                                                                   \
               head_val[off_ + k_] = acc[k_];                                                   \
               if(MODE == kLse) head_aux[off_ + k_] = aux[k_];                                  \
            }                                                                                   \
         } else {                                                                               \
            A fin_[VN];                                                                         \
            _Pragma("unroll") for(int k_ = 0; k_ < VN; ++k_) fin_[k_] =                         \
               (MODE == kLse) ? lse_value(acc[k_], aux[k_], LF) : acc[k_];                      \
            if(PF) {                                                                            \
               epi_finish((R_), cnt_, fin_);                                                    \
            } else if(MODE == kSumEpi) {                                                        \
               epi_apply< T, VN >(p, (R_), col, fin_);                                           \
            }                                                                                   \
            store_chunk< T, PB >(out + (int64_t)(R_)*p.emb + col, fin_);                         \
         }                                                                                      \
      }                                                                                         \
      if(head_) head_row = (R_);                                                                \
      RELM_MP_STREAM_RESET();                                                                   \
   } while(0)

#pragma unroll
      for(int s = 0; s < kStreamStages - 1; ++s) issue(s);
      RELM_MP_STREAM_RESET();
      int R = r_begin;
      int rend = (R < r_end) ? row_end(R) : INT_MAX;
      int own_row = -1;
      bool pending = false;
      for(int k = 0; k < nbatches; ++k) {
         issue(k + kStreamStages - 1);
         cp_async_wait< kStreamStages - 1 >();
         __syncwarp();
         const int j0 = j_begin + k * B;
         const int nb = (j_end - j0) < B ? (j_end - j0) : B;
         const unsigned char* st = wbase + (k % kStreamStages) * kStreamStageBytes;
         int b = 0;
         while(b < nb) {
            while(rend <= j0 + b) {
               RELM_MP_STREAM_FLUSH(R, rend);
               ++R;
               rend = (R < r_end) ? row_end(R) : INT_MAX;
            }
            // Edges [b, b + run) of this batch all belong to the open row R.
            const int run = (nb - b) < (rend - (j0 + b)) ? (nb - b) : (rend - (j0 + b));
            if(lane_ok) {
               const unsigned char* src = st + b * CBW + lane * PB;
               if(MODE == kLseBwd) {
                  if(own_row != R) {
                     load_chunk_global< T, PB >(own + (int64_t)R * p.emb + col, ownv);
                     own_row = R;
                  }
                  for(int q = 0; q < run; ++q) {
                     A v[VN], w[VN];
                     load_chunk< T, PB >(reinterpret_cast< const T* >(src + q * CBW), v);
                     load_chunk< T, PB >(
                        reinterpret_cast< const T* >(src + kStreamStages * kStreamStageBytes + q * CBW), w
                     );
#pragma unroll
                     for(int x = 0; x < VN; ++x) acc[x] += v[x] * exp_k(ownv[x] - w[x], LF.k);
                  }
               } else if constexpr(kPairs) {
                  // folds of 8, then 4, then the last 1..3 edges of the run (one rescale each)
                  auto fold = [&](auto width, int q0, int nval) __attribute__((always_inline)) {
                     constexpr int N = decltype(width)::value;
                     if constexpr(sizeof(T) == 2 && MODE == kLse && PB == 4) {
                        // one packed pair per edge straight from shared memory (wider
                        // lane chunks keep the float path: their eight-edge folds
                        // would not fit the registers)
                        constexpr int NW = PB / 4;
                        uint32_t w[N][NW];
#pragma unroll
                        for(int i = 0; i < N; ++i) {
#pragma unroll
                           for(int j = 0; j < NW; ++j)
                              w[i][j] = i < nval ? reinterpret_cast< const uint32_t* >(src + (q0 + i) * CBW)[j]
                                                 : kNegInf2< T >;
                        }
#pragma unroll
                        for(int j = 0; j < NW; ++j) {
                           uint32_t wj[N];
#pragma unroll
                           for(int i = 0; i < N; ++i) wj[i] = w[i][j];
                           float2 a = make_float2(acc[2 * j], acc[2 * j + 1]);
                           float2 sx = make_float2(aux[2 * j], aux[2 * j + 1]);
                           lse_fold2_packed< T, N >(a, sx, wj, nval, LF.k);
                           acc[2 * j] = a.x;
                           acc[2 * j + 1] = a.y;
                           aux[2 * j] = sx.x;
                           aux[2 * j + 1] = sx.y;
                        }
                     } else {
                        A v[N][VN];
#pragma unroll
                        for(int i = 0; i < N; ++i) {
                           if(i < nval) {
                              load_chunk< T, PB >(reinterpret_cast< const T* >(src + (q0 + i) * CBW), v[i]);
                           } else {
#pragma unroll
                              for(int x = 0; x < VN; ++x) v[i][x] = (sum_mode(MODE)) ? A(0) : ninf;
                           }
                        }
#pragma unroll
                        for(int x = 0; x < VN; x += 2) {
                           float2 vx[N];
#pragma unroll
                           for(int i = 0; i < N; ++i) vx[i] = make_float2(v[i][x], v[i][x + 1]);
                           float2 a = make_float2(acc[x], acc[x + 1]);
                           if(sum_mode(MODE)) {
#pragma unroll
                              for(int w = 1; w < N; w <<= 1)
#pragma unroll
                                 for(int i = 0; i + w < N; i += 2 * w) vx[i] = add2(vx[i], vx[i + w]);
                              a = add2(a, vx[0]);
                           } else {
                              float2 sx = make_float2(aux[x], aux[x + 1]);
                              lse_fold2< N >(a, sx, vx, nval, LF.k);
                              aux[x] = sx.x;
                              aux[x + 1] = sx.y;
                           }
                           acc[x] = a.x;
                           acc[x + 1] = a.y;
                        }
                     }
                  };
                  // lanes of two columns fold 8 edges at a time; wider lane chunks 4
                  // (their eight-edge folds would not fit the registers)
                  int q = 0;
                  if constexpr(VN <= 2)
                     for(; q + 8 <= run; q += 8) fold(std::integral_constant< int, 8 >{}, q, 8);
                  for(; q + 4 <= run; q += 4) fold(std::integral_constant< int, 4 >{}, q, 4);
                  if(q < run) fold(std::integral_constant< int, 3 >{}, q, run - q);
               } else {
                  int q = 0;
                  for(; q + 4 <= run; q += 4) {
                     A v[4][VN];
#pragma unroll
                     for(int i = 0; i < 4; ++i)
                        load_chunk< T, PB >(reinterpret_cast< const T* >(src + (q + i) * CBW), v[i]);
#pragma unroll
                     for(int x = 0; x < VN; ++x) {
                        if(sum_mode(MODE)) {
                           acc[x] += v[0][x] + v[1][x] + v[2][x] + v[3][x];
                        } else {
                           const A vx[4] = {v[0][x], v[1][x], v[2][x], v[3][x]};
                           lse_fold< A, 4 >(acc[x], aux[x], vx, 4, LF.k);
                        }
                     }
                  }
                  if(q < run) {  // the last 1..3 edges of the run as one fold (one rescale)
                     const int rem = run - q;
                     A v[3][VN];
#pragma unroll
                     for(int i = 0; i < 3; ++i) {
                        if(i < rem) {
                           load_chunk< T, PB >(reinterpret_cast< const T* >(src + (q + i) * CBW), v[i]);
                        } else {
#pragma unroll
                           for(int x = 0; x < VN; ++x) v[i][x] = (sum_mode(MODE)) ? A(0) : ninf;
                        }
                     }
#pragma unroll
                     for(int x = 0; x < VN; ++x) {
                        if(sum_mode(MODE)) {
                           acc[x] += v[0][x] + v[1][x] + v[2][x];
                        } else {
                           const A vx[3] = {v[0][x], v[1][x], v[2][x]};
                           lse_fold< A, 3 >(acc[x], aux[x], vx, rem, LF.k);
                        }
                     }
                  }
               }
            }
            b += run;
         }
         pending = true;
         __syncwarp();
      }
      cp_async_wait< 0 >();
      if(R < r_end) pending = false;
      while(R < r_end) {
         RELM_MP_STREAM_FLUSH(R, row_end(R));
         ++R;
      }
#undef RELM_MP_STREAM_FLUSH
#undef RELM_MP_STREAM_RESET
      if(pending) {
         if constexpr(kFloor) {
#pragma unroll
            for(int k = 0; k < VN; ++k) lse_floor_fix(acc[k], aux[k], j_end - e_rstart);
         }
         if(lane_ok) {
            const int64_t off = tile * p.emb + col;
#pragma unroll
            for(int k = 0; k < VN; ++k) {
               tail_val[off + k] = acc[k];
               if(MODE == kLse) tail_aux[off + k] = aux[k];
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
// F independent loads in flight (8; kLongFold in the long-row fixup).
template < typename T, int MODE, int F = 8 >
__device__ __forceinline__ void fixup_combine(const SegParams& p, int64_t t_first, int64_t t_last, int64_t col,
                                              typename AccOf< T >::type& m, typename AccOf< T >::type& s)
{
   using A = typename AccOf< T >::type;
   const A* tail_val = static_cast< const A* >(p.tail_val);
   const A* tail_aux = static_cast< const A* >(p.tail_aux);
   const A k = (A)p.lse_k;
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
            lse_merge(m, s, a[i], b[i], k);
         else
            m += a[i];
      }
   }
   for(; u < t_last; ++u) {
      const int64_t off = u * p.emb + col;
      if(MODE == kLse)
         lse_merge(m, s, tail_val[off], tail_aux[off], k);
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
      const LseForm< A > LF = lse_form< A >(p);
      lse_merge(m, s, head_val[off], head_aux[off], LF.k);
      res = lse_value(m, s, LF);
   } else {
      res = m + head_val[off];
      if(MODE == kSumEpi) {
         A one[1] = {res};
         epi_apply< T, 1 >(p, R, col, one);
         res = one[0];
      }
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
   if(t >= p.num_tiles || !merge_path_runs(p)) return;
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
constexpr int kLongFold = 16;  // partials in flight per lane in the long-row fixup (latency-bound)

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
   if(!merge_path_runs(p)) return;
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
      if(col < p.emb && u0 < u1) fixup_combine< T, MODE, kLongFold >(p, u0, u1, col, m, s);
      sm_m[warp][lane] = m;
      sm_s[warp][lane] = s;
      __syncthreads();
      if(warp == 0 && col < p.emb) {
         A mm = sm_m[0][lane];
         A ss = sm_s[0][lane];
         for(int w = 1; w < W; ++w) {
            if(MODE == kLse)
               lse_merge(mm, ss, sm_m[w][lane], sm_s[w][lane], (A)p.lse_k);
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
int launch_row_map(const SegParams& p, int mode, int vb, int chmax, cudaStream_t stream);
template < typename T >
int launch_seg_reduce(const SegParams& pm, int vb_map, int ch_map, const SegParams& p, int vb, int chmax, int mode,
                      cudaStream_t stream);
template < typename T >
int launch_scatter_lse_bwd(const SegParams& p, const uint32_t* cover, int64_t out_rows, cudaStream_t stream);
template < typename T >
int launch_scatter_rows(const SegParams& p, const uint32_t* cover, int64_t out_rows, int vb, int chmax,
                        cudaStream_t stream);
// Shared-memory pipeline variant (rows of 16-byte multiples, 16-byte aligned):
// pb = bytes per lane, p.block_cols = column block in elements, p.ch = rows per stage.
template < typename T >
int launch_seg_stream(const SegParams& pm, int vb_map, int ch_map, const SegParams& p, int pb, int mode,
                      cudaStream_t stream);

}  // namespace relm_mp
