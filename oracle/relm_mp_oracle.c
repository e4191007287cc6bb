/*
 * CPU oracle for the relm_mp fan-out / fan-in path.
 *
 * TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg use this file as the checker. The relmo_b200 product never
 * links, loads or calls it.
 *
 * A plain-C restatement of the reference's CPU semantics (maichmueller/relmo,
 * src/_ops/mp/mp_ops.cpp):
 *   - fanout_scatter            : CPU loop      mp_ops.cpp:2815-2836
 *   - fanout_scatter_backward   : CPU loop      mp_ops.cpp:2838-2861
 *   - fanin_reduce (sum)        : CPU loop      mp_ops.cpp:2863-2886
 *   - fanin_reduce_sum_backward : CPU loop      mp_ops.cpp:2888-2911
 *   - fanin_reduce (logsumexp)  : ATen formula  mp_ops.cpp:3005-3036
 *       (amax scatter-reduce, exp(x - max), scatter-add, log(sum) + max)
 *   - fanin_reduce_logsumexp_backward : ATen formula mp_ops.cpp:2981-3003
 *       (grad_rel[src] += grad_out[dst] * exp(rel[src] - out[dst]))
 * Arithmetic happens in the element type (float or double), in edge order, as
 * in the reference loops. bf16 inputs are checked against the float oracle on
 * upcast inputs (the reference has no bf16 accumulation kernel).
 *
 * Every function returns 0 on success or the 1-based number of the index array
 * that held the first out-of-range value (1 = first index argument, 2 =
 * second), with *bad_pos set to the edge position and *bad_value to the value.
 * The reference raises at the same first offending edge (mp_ops.cpp:59-64,
 * 2830-2831).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ORACLE_EXPORT __attribute__((visibility("default")))

static int check_pair(const int64_t* a, int64_t a_size, const int64_t* b, int64_t b_size,
                      int64_t e, int64_t* bad_pos, int64_t* bad_value)
{
   if(a[e] < 0 || a[e] >= a_size) {
      *bad_pos = e;
      *bad_value = a[e];
      return 1;
   }
   if(b[e] < 0 || b[e] >= b_size) {
      *bad_pos = e;
      *bad_value = b[e];
      return 2;
   }
   return 0;
}

#define DEFINE_ORACLE(T, SUFFIX, EXP, LOG)                                                      \
   /* mp_ops.cpp:2815-2836: out = zeros; out[flat_dst[e]] = x[src[e]] (last writer wins). */   \
   ORACLE_EXPORT int relm_oracle_fanout_scatter_##SUFFIX(                                      \
      const T* x, int64_t x_rows, int64_t emb, const int64_t* src, const int64_t* flat_dst,    \
      int64_t num_edges, int64_t out_rows, T* out, int64_t* bad_pos, int64_t* bad_value)       \
   {                                                                                            \
      memset(out, 0, (size_t)(out_rows * emb) * sizeof(T));                                    \
      if(num_edges == 0 || out_rows == 0) return 0;                                            \
      for(int64_t e = 0; e < num_edges; ++e) {                                                 \
         int rc = check_pair(src, x_rows, flat_dst, out_rows, e, bad_pos, bad_value);          \
         if(rc) return rc;                                                                      \
         memcpy(out + flat_dst[e] * emb, x + src[e] * emb, (size_t)emb * sizeof(T));           \
      }                                                                                         \
      return 0;                                                                                 \
   }                                                                                            \
   /* mp_ops.cpp:2838-2861: grad_x = zeros; grad_x[src[e]] += grad_out[flat_dst[e]]. */       \
   ORACLE_EXPORT int relm_oracle_fanout_scatter_backward_##SUFFIX(                             \
      const T* grad_out, int64_t grad_out_rows, int64_t emb, const int64_t* src,               \
      const int64_t* flat_dst, int64_t num_edges, int64_t x_rows, T* grad_x, int64_t* bad_pos, \
      int64_t* bad_value)                                                                       \
   {                                                                                            \
      memset(grad_x, 0, (size_t)(x_rows * emb) * sizeof(T));                                   \
      if(num_edges == 0 || x_rows == 0) return 0;                                              \
      for(int64_t e = 0; e < num_edges; ++e) {                                                 \
         int rc = check_pair(src, x_rows, flat_dst, grad_out_rows, e, bad_pos, bad_value);     \
         if(rc) return rc;                                                                      \
         const T* in = grad_out + flat_dst[e] * emb;                                           \
         T* o = grad_x + src[e] * emb;                                                          \
         for(int64_t k = 0; k < emb; ++k) o[k] += in[k];                                       \
      }                                                                                         \
      return 0;                                                                                 \
   }                                                                                            \
   /* mp_ops.cpp:2863-2886: out = zeros; out[dst[e]] += rel[flat_src[e]]. */                   \
   ORACLE_EXPORT int relm_oracle_fanin_sum_##SUFFIX(                                           \
      const T* rel, int64_t rel_rows, int64_t emb, const int64_t* flat_src,                    \
      const int64_t* dst, int64_t num_edges, int64_t dim_size, T* out, int64_t* bad_pos,       \
      int64_t* bad_value)                                                                       \
   {                                                                                            \
      memset(out, 0, (size_t)(dim_size * emb) * sizeof(T));                                   \
      if(num_edges == 0 || dim_size == 0) return 0;                                            \
      for(int64_t e = 0; e < num_edges; ++e) {                                                 \
         int rc = check_pair(flat_src, rel_rows, dst, dim_size, e, bad_pos, bad_value);        \
         if(rc) return rc;                                                                      \
         const T* in = rel + flat_src[e] * emb;                                                \
         T* o = out + dst[e] * emb;                                                             \
         for(int64_t k = 0; k < emb; ++k) o[k] += in[k];                                       \
      }                                                                                         \
      return 0;                                                                                 \
   }                                                                                            \
   /* mp_ops.cpp:2888-2911: grad_rel = zeros; grad_rel[flat_src[e]] += grad_out[dst[e]]. */    \
   ORACLE_EXPORT int relm_oracle_fanin_sum_backward_##SUFFIX(                                  \
      const T* grad_out, int64_t grad_out_rows, int64_t emb, const int64_t* flat_src,          \
      const int64_t* dst, int64_t num_edges, int64_t rel_rows, T* grad_rel, int64_t* bad_pos,  \
      int64_t* bad_value)                                                                       \
   {                                                                                            \
      memset(grad_rel, 0, (size_t)(rel_rows * emb) * sizeof(T));                               \
      if(num_edges == 0 || rel_rows == 0) return 0;                                            \
      for(int64_t e = 0; e < num_edges; ++e) {                                                 \
         int rc = check_pair(flat_src, rel_rows, dst, grad_out_rows, e, bad_pos, bad_value);   \
         if(rc) return rc;                                                                      \
         const T* in = grad_out + dst[e] * emb;                                                \
         T* o = grad_rel + flat_src[e] * emb;                                                   \
         for(int64_t k = 0; k < emb; ++k) o[k] += in[k];                                       \
      }                                                                                         \
      return 0;                                                                                 \
   }                                                                                            \
   /* mp_ops.cpp:3005-3036 (ATen path): amax per (row, column) with NaN propagation,        \
    * then sum of exp(x - amax), then log(sum) + amax. Empty rows stay -inf.                  \
    * amax_scratch and sum_scratch are caller-provided [dim_size * emb]. */                   \
   ORACLE_EXPORT int relm_oracle_fanin_logsumexp_##SUFFIX(                                     \
      const T* rel, int64_t rel_rows, int64_t emb, const int64_t* flat_src,                    \
      const int64_t* dst, int64_t num_edges, int64_t dim_size, T* out, T* sum_scratch,         \
      int64_t* bad_pos, int64_t* bad_value)                                                    \
   {                                                                                            \
      const int64_t n = dim_size * emb;                                                        \
      for(int64_t i = 0; i < n; ++i) out[i] = (T)(-INFINITY);                                  \
      if(num_edges == 0 || dim_size == 0) return 0;                                            \
      for(int64_t e = 0; e < num_edges; ++e) {                                                 \
         int rc = check_pair(flat_src, rel_rows, dst, dim_size, e, bad_pos, bad_value);        \
         if(rc) return rc;                                                                      \
      }                                                                                         \
      T* amax = out;                                                                            \
      for(int64_t e = 0; e < num_edges; ++e) {                                                 \
         const T* in = rel + flat_src[e] * emb;                                                \
         T* m = amax + dst[e] * emb;                                                            \
         for(int64_t k = 0; k < emb; ++k) {                                                    \
            if(isnan(in[k]) || in[k] > m[k]) m[k] = in[k];                                     \
         }                                                                                      \
      }                                                                                         \
      memset(sum_scratch, 0, (size_t)n * sizeof(T));                                           \
      for(int64_t e = 0; e < num_edges; ++e) {                                                 \
         const T* in = rel + flat_src[e] * emb;                                                \
         const T* m = amax + dst[e] * emb;                                                      \
         T* s = sum_scratch + dst[e] * emb;                                                     \
         for(int64_t k = 0; k < emb; ++k) s[k] += EXP(in[k] - m[k]);                           \
      }                                                                                         \
      for(int64_t i = 0; i < n; ++i) out[i] = LOG(sum_scratch[i]) + amax[i];                   \
      return 0;                                                                                 \
   }                                                                                            \
   /* mp_ops.cpp:2981-3003 (ATen fallback): grad_rel = zeros;                                 \
    * grad_rel[flat_src[e]] += grad_out[dst[e]] * exp(rel[flat_src[e]] - out[dst[e]]). */      \
   ORACLE_EXPORT int relm_oracle_fanin_logsumexp_backward_##SUFFIX(                            \
      const T* grad_out, const T* rel, const T* out, int64_t dim_size, int64_t emb,            \
      const int64_t* flat_src, const int64_t* dst, int64_t num_edges, int64_t rel_rows,        \
      T* grad_rel, int64_t* bad_pos, int64_t* bad_value)                                       \
   {                                                                                            \
      memset(grad_rel, 0, (size_t)(rel_rows * emb) * sizeof(T));                               \
      if(num_edges == 0 || rel_rows == 0) return 0;                                            \
      for(int64_t e = 0; e < num_edges; ++e) {                                                 \
         int rc = check_pair(flat_src, rel_rows, dst, dim_size, e, bad_pos, bad_value);        \
         if(rc) return rc;                                                                      \
      }                                                                                         \
      for(int64_t e = 0; e < num_edges; ++e) {                                                 \
         const T* g = grad_out + dst[e] * emb;                                                 \
         const T* o = out + dst[e] * emb;                                                       \
         const T* r = rel + flat_src[e] * emb;                                                  \
         T* gr = grad_rel + flat_src[e] * emb;                                                  \
         for(int64_t k = 0; k < emb; ++k) gr[k] += g[k] * EXP(r[k] - o[k]);                    \
      }                                                                                         \
      return 0;                                                                                 \
   }

DEFINE_ORACLE(float, f32, expf, logf)
DEFINE_ORACLE(double, f64, exp, log)
