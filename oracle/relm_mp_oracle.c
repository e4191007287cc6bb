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
 *   - LGAN ops, sum / mean modes : ATen formulas
 *       lgan_pool_reduce mp_ops.cpp:3424-3469, lgan_pool_reduce_backward
 *       3527-3572, lgan_relation_graph_step 3627-3656,
 *       lgan_relation_graph_step_backward 3715-3743; one indexed sum / mean
 *       is relmo/ops/mp_common.py:88-118 (index_select, index_add_ in edge
 *       order, then a division by max(count, 1) in the element type).
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
#include <stdlib.h>
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

/* Index checks of the LGAN formulas: index_select checks its index before
 * index_add_ checks its own, each at its first offending position. Return
 * codes name the index array: 1 rr_src, 2 rr_dst, 3 tn_rel, 4 tn_ent, 5 nn_rel,
 * 6 nn_ent, 7 slot_to_relation_instance. */
static int check_index(const int64_t* a, int64_t n, int64_t bound, int code, int64_t* bad_pos, int64_t* bad_value)
{
   for(int64_t e = 0; e < n; ++e) {
      if(a[e] < 0 || a[e] >= bound) {
         *bad_pos = e;
         *bad_value = a[e];
         return code;
      }
   }
   return 0;
}

#define DEFINE_LGAN(T, SUFFIX)                                                                       \
   /* agg(x, src -> dst, rows): zeros, index_add_ of x[src] at dst, mean: / max(count, 1)           \
    * (mp_common.py:88-118; mp_ops.cpp:3433-3454). */                                               \
   static int lgan_agg_##SUFFIX(const T* x, int64_t x_rows, int64_t emb, const int64_t* src,         \
                                const int64_t* dst, int64_t n, int64_t rows, int mean, T* out,       \
                                int src_code, int dst_code, int64_t* bad_pos, int64_t* bad_value)    \
   {                                                                                                 \
      memset(out, 0, (size_t)(rows * emb) * sizeof(T));                                             \
      if(n == 0 || rows == 0) return 0;                                                             \
      int rc = check_index(src, n, x_rows, src_code, bad_pos, bad_value);                           \
      if(rc) return rc;                                                                              \
      if((rc = check_index(dst, n, rows, dst_code, bad_pos, bad_value))) return rc;                 \
      for(int64_t e = 0; e < n; ++e) {                                                              \
         const T* in = x + src[e] * emb;                                                            \
         T* o = out + dst[e] * emb;                                                                  \
         for(int64_t k = 0; k < emb; ++k) o[k] += in[k];                                            \
      }                                                                                              \
      if(mean) {                                                                                     \
         T* cnt = (T*)calloc((size_t)rows, sizeof(T));                                              \
         for(int64_t e = 0; e < n; ++e) cnt[dst[e]] += (T)1;                                        \
         for(int64_t r = 0; r < rows; ++r) {                                                        \
            const T d = cnt[r] > (T)1 ? cnt[r] : (T)1;                                              \
            for(int64_t k = 0; k < emb; ++k) out[r * emb + k] = out[r * emb + k] / d;               \
         }                                                                                           \
         free(cnt);                                                                                  \
      }                                                                                              \
      return 0;                                                                                      \
   }                                                                                                 \
   /* The reverse (mp_ops.cpp:3527-3555): zeros [rows]; gathered = g[dst] (mean: / max(count of   \
    * dst over g's rows, 1)); index_add_ at src. */                                                 \
   static int lgan_rev_##SUFFIX(const T* g, int64_t g_rows, int64_t emb, const int64_t* src,         \
                                const int64_t* dst, int64_t n, int64_t rows, int mean, T* out,       \
                                int src_code, int dst_code, int64_t* bad_pos, int64_t* bad_value)    \
   {                                                                                                 \
      memset(out, 0, (size_t)(rows * emb) * sizeof(T));                                             \
      if(n == 0 || rows == 0) return 0;                                                             \
      int rc = check_index(dst, n, g_rows, dst_code, bad_pos, bad_value);                           \
      if(rc) return rc;                                                                              \
      if((rc = check_index(src, n, rows, src_code, bad_pos, bad_value))) return rc;                 \
      T* cnt = NULL;                                                                                 \
      if(mean) {                                                                                     \
         cnt = (T*)calloc((size_t)(g_rows > 0 ? g_rows : 1), sizeof(T));                            \
         for(int64_t e = 0; e < n; ++e) cnt[dst[e]] += (T)1;                                        \
      }                                                                                              \
      for(int64_t e = 0; e < n; ++e) {                                                              \
         const T* in = g + dst[e] * emb;                                                            \
         T* o = out + src[e] * emb;                                                                  \
         const T d = mean ? (cnt[dst[e]] > (T)1 ? cnt[dst[e]] : (T)1) : (T)1;                       \
         for(int64_t k = 0; k < emb; ++k) o[k] += mean ? in[k] / d : in[k];                         \
      }                                                                                              \
      free(cnt);                                                                                     \
      return 0;                                                                                      \
   }                                                                                                 \
   /* mp_ops.cpp:3627-3656: x1 = x + agg(x, rr); tn = agg(x1, tn); nn = agg(x1, nn). */             \
   ORACLE_EXPORT int relm_oracle_lgan_relation_graph_step_##SUFFIX(                                 \
      const T* x, int64_t rows, int64_t emb, const int64_t* rr_src, const int64_t* rr_dst,          \
      int64_t n_rr, const int64_t* tn_rel, const int64_t* tn_ent, int64_t n_tn,                     \
      const int64_t* nn_rel, const int64_t* nn_ent, int64_t n_nn, int64_t entity_dim_size,          \
      int mean, T* x_out, T* tn, T* nn, int64_t* bad_pos, int64_t* bad_value)                       \
   {                                                                                                 \
      int rc = lgan_agg_##SUFFIX(x, rows, emb, rr_src, rr_dst, n_rr, rows, mean, x_out, 1, 2,       \
                                 bad_pos, bad_value);                                                \
      if(rc) return rc;                                                                              \
      for(int64_t i = 0; i < rows * emb; ++i) x_out[i] = x[i] + x_out[i];                          \
      if((rc = lgan_agg_##SUFFIX(x_out, rows, emb, tn_rel, tn_ent, n_tn, entity_dim_size, mean, tn, \
                                 3, 4, bad_pos, bad_value)))                                         \
         return rc;                                                                                  \
      return lgan_agg_##SUFFIX(x_out, rows, emb, nn_rel, nn_ent, n_nn, entity_dim_size, mean, nn,   \
                               5, 6, bad_pos, bad_value);                                            \
   }                                                                                                 \
   /* mp_ops.cpp:3715-3743: g = gx + rev(gtn, tn) + rev(gnn, nn); return g + rev(g, rr). */         \
   ORACLE_EXPORT int relm_oracle_lgan_relation_graph_step_backward_##SUFFIX(                        \
      const T* gx, const T* gtn, const T* gnn, int64_t entity_rows, int64_t emb,                    \
      const int64_t* rr_src, const int64_t* rr_dst, int64_t n_rr, const int64_t* tn_rel,           \
      const int64_t* tn_ent, int64_t n_tn, const int64_t* nn_rel, const int64_t* nn_ent,            \
      int64_t n_nn, int64_t relation_count, int mean, T* grad_x, int64_t* bad_pos,                  \
      int64_t* bad_value)                                                                            \
   {                                                                                                 \
      const int64_t n = relation_count * emb;                                                       \
      T* a = (T*)malloc((size_t)(n > 0 ? n : 1) * sizeof(T));                                       \
      T* g = (T*)calloc((size_t)(n > 0 ? n : 1), sizeof(T));                                        \
      int rc = lgan_rev_##SUFFIX(gtn, entity_rows, emb, tn_rel, tn_ent, n_tn, relation_count, mean, \
                                 a, 3, 4, bad_pos, bad_value);                                      \
      if(!rc) {                                                                                      \
         for(int64_t i = 0; i < n; ++i) g[i] = gx[i] + a[i];                                        \
         rc = lgan_rev_##SUFFIX(gnn, entity_rows, emb, nn_rel, nn_ent, n_nn, relation_count, mean,  \
                                a, 5, 6, bad_pos, bad_value);                                       \
      }                                                                                              \
      if(!rc) {                                                                                      \
         for(int64_t i = 0; i < n; ++i) g[i] = g[i] + a[i];                                         \
         rc = lgan_rev_##SUFFIX(g, relation_count, emb, rr_src, rr_dst, n_rr, relation_count, mean, \
                                a, 1, 2, bad_pos, bad_value);                                       \
      }                                                                                              \
      if(!rc)                                                                                        \
         for(int64_t i = 0; i < n; ++i) grad_x[i] = g[i] + a[i];                                    \
      free(a);                                                                                       \
      free(g);                                                                                       \
      return rc;                                                                                     \
   }                                                                                                 \
   /* mp_ops.cpp:3424-3469: x0 = index_add_ of the slots / max(arity, 1), then the graph step. */   \
   ORACLE_EXPORT int relm_oracle_lgan_pool_reduce_##SUFFIX(                                         \
      const T* slots, int64_t num_slots, int64_t emb, const int64_t* slot_to_rel,                   \
      const int64_t* arities, int64_t relation_count, const int64_t* rr_src, const int64_t* rr_dst, \
      int64_t n_rr, const int64_t* tn_rel, const int64_t* tn_ent, int64_t n_tn,                     \
      const int64_t* nn_rel, const int64_t* nn_ent, int64_t n_nn, int64_t entity_dim_size,          \
      int mean, T* x_out, T* tn, T* nn, int64_t* bad_pos, int64_t* bad_value)                       \
   {                                                                                                 \
      const int64_t n = relation_count * emb;                                                       \
      T* x0 = (T*)calloc((size_t)(n > 0 ? n : 1), sizeof(T));                                       \
      int rc = 0;                                                                                    \
      if(num_slots * emb > 0) {                                                                      \
         rc = check_index(slot_to_rel, num_slots, relation_count, 7, bad_pos, bad_value);           \
         if(!rc) {                                                                                   \
            for(int64_t s = 0; s < num_slots; ++s)                                                  \
               for(int64_t k = 0; k < emb; ++k) x0[slot_to_rel[s] * emb + k] += slots[s * emb + k]; \
            for(int64_t r = 0; r < relation_count; ++r) {                                           \
               const T a = (T)arities[r];                                                           \
               const T d = a > (T)1 ? a : (T)1;                                                     \
               for(int64_t k = 0; k < emb; ++k) x0[r * emb + k] = x0[r * emb + k] / d;              \
            }                                                                                        \
         }                                                                                           \
      }                                                                                              \
      if(!rc)                                                                                        \
         rc = relm_oracle_lgan_relation_graph_step_##SUFFIX(                                        \
            x0, relation_count, emb, rr_src, rr_dst, n_rr, tn_rel, tn_ent, n_tn, nn_rel, nn_ent,    \
            n_nn, entity_dim_size, mean, x_out, tn, nn, bad_pos, bad_value);                        \
      free(x0);                                                                                      \
      return rc;                                                                                     \
   }                                                                                                 \
   /* mp_ops.cpp:3527-3572: the graph-step backward, then grad_slot = g[s2r] / max(arity[s2r], 1). */\
   ORACLE_EXPORT int relm_oracle_lgan_pool_reduce_backward_##SUFFIX(                                \
      const T* gx, const T* gtn, const T* gnn, int64_t entity_rows, int64_t emb,                    \
      const int64_t* slot_to_rel, int64_t num_slots, const int64_t* arities, const int64_t* rr_src, \
      const int64_t* rr_dst, int64_t n_rr, const int64_t* tn_rel, const int64_t* tn_ent,           \
      int64_t n_tn, const int64_t* nn_rel, const int64_t* nn_ent, int64_t n_nn,                     \
      int64_t relation_count, int mean, T* grad_slots, int64_t* bad_pos, int64_t* bad_value)        \
   {                                                                                                 \
      const int64_t n = relation_count * emb;                                                       \
      T* g = (T*)malloc((size_t)(n > 0 ? n : 1) * sizeof(T));                                       \
      int rc = relm_oracle_lgan_relation_graph_step_backward_##SUFFIX(                              \
         gx, gtn, gnn, entity_rows, emb, rr_src, rr_dst, n_rr, tn_rel, tn_ent, n_tn, nn_rel,        \
         nn_ent, n_nn, relation_count, mean, g, bad_pos, bad_value);                                \
      if(!rc) rc = check_index(slot_to_rel, num_slots, relation_count, 7, bad_pos, bad_value);      \
      if(!rc) {                                                                                      \
         for(int64_t s = 0; s < num_slots; ++s) {                                                   \
            const T a = (T)arities[slot_to_rel[s]];                                                 \
            const T d = a > (T)1 ? a : (T)1;                                                        \
            for(int64_t k = 0; k < emb; ++k) grad_slots[s * emb + k] = g[slot_to_rel[s] * emb + k] / d; \
         }                                                                                           \
      }                                                                                              \
      free(g);                                                                                       \
      return rc;                                                                                     \
   }

DEFINE_LGAN(float, f32)
DEFINE_LGAN(double, f64)
