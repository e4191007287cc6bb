// CPU kernels of torch.ops.relm_mp, registered under the CPU dispatch key.
//
// The reference library registers its ops for every backend
// (CompositeImplicitAutograd, mp_ops.cpp:3840-3911), so relmo's facade sends
// CPU tensors to the custom op whenever the library loads
// (relmo/ops/mp.py:49-51, 65-68). This library must take them too, with the
// reference CPU library's results and errors:
//   - float32 / float64 fan-out, fan-out backward, fan-in sum and its backward
//     are loops in edge order with a bounds check per edge (first the gathered
//     index, then the written one, as mp_ops.cpp:2815-2911 checks them), so the
//     sums add in the reference's order and come out bit-identical;
//   - other dtypes, logsumexp and its backward, and the LGAN ops evaluate the
//     reference's ATen formulas (mp_ops.cpp:2913-3036, 3424-3469, 3527-3572,
//     3627-3656, 3715-3743); ATen raises its own errors for bad indices there,
//     as in the reference.
// Argument checks and their messages are those of the CUDA registration
// (relm_mp_torch.cpp), which follow mp_ops.cpp.
#include <ATen/ATen.h>
#include <torch/library.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <tuple>

#include "relm_mp_torch.h"

namespace relm_b200 {
namespace {

using at::Tensor;

constexpr int64_t kModeSum = 0;
constexpr int64_t kModeLogSumExp = 1;
constexpr int64_t kModeMean = 2;

inline void check_bound(int64_t v, int64_t n, const char* name)
{
   TORCH_CHECK(v >= 0 && v < n, name, " index out of bounds: ", v, " not in [0, ", n, ").");
}

bool loop_dtype(const Tensor& t) { return t.scalar_type() == at::kFloat || t.scalar_type() == at::kDouble; }

// out[dst[e]] = x[src[e]] for e in order: a repeated slot keeps the last edge.
template < typename T >
void copy_rows(const T* x, int64_t x_rows, const int64_t* src, const int64_t* dst, int64_t edges, int64_t out_rows,
               int64_t emb, T* out)
{
   for(int64_t e = 0; e < edges; ++e) {
      check_bound(src[e], x_rows, "src_global_idx");
      check_bound(dst[e], out_rows, "flat_dst");
      std::memcpy(out + dst[e] * emb, x + src[e] * emb, (size_t)emb * sizeof(T));
   }
}

// For e in order: out[w[e]] += in[r[e]], where `first` (checked first) is w
// when write_first, else r.
template < typename T >
void add_rows(const T* in, const int64_t* r, int64_t in_rows, const char* r_name, T* out, const int64_t* w,
              int64_t out_rows, const char* w_name, bool write_first, int64_t edges, int64_t emb)
{
   for(int64_t e = 0; e < edges; ++e) {
      if(write_first) {
         check_bound(w[e], out_rows, w_name);
         check_bound(r[e], in_rows, r_name);
      } else {
         check_bound(r[e], in_rows, r_name);
         check_bound(w[e], out_rows, w_name);
      }
      const T* a = in + r[e] * emb;
      T* o = out + w[e] * emb;
      for(int64_t k = 0; k < emb; ++k) o[k] += a[k];
   }
}

template < typename F >
void float_or_double(const Tensor& t, F&& f)
{
   if(t.scalar_type() == at::kFloat)
      f(float{});
   else
      f(double{});
}

// ---- the hot ops ---------------------------------------------------------------

// mp_ops.cpp:3038-3101 (loop 2815-2836, fallback 2913-2928)
Tensor fanout_scatter_cpu(const Tensor& x_cat, const Tensor& src_global_idx, const Tensor& flat_dst, int64_t out_rows)
{
   check_rank(x_cat, 2, "x_cat");
   check_int64_index(src_global_idx, "src_global_idx");
   check_int64_index(flat_dst, "flat_dst");
   TORCH_CHECK(src_global_idx.size(0) == flat_dst.size(0), "src_global_idx and flat_dst must have equal length.");
   TORCH_CHECK(out_rows >= 0, "out_rows must be >= 0.");
   const int64_t emb = x_cat.size(1);
   Tensor out = at::zeros({out_rows, emb}, x_cat.options());
   if(src_global_idx.numel() == 0 || out_rows == 0) return out;
   if(!loop_dtype(x_cat)) {
      out.index_copy_(0, flat_dst, x_cat.index_select(0, src_global_idx));
      return out;
   }
   const Tensor x = contig(x_cat), src = contig(src_global_idx), dst = contig(flat_dst);
   float_or_double(x, [&](auto v) {
      using T = decltype(v);
      copy_rows< T >(x.data_ptr< T >(), x.size(0), src.data_ptr< int64_t >(), dst.data_ptr< int64_t >(), src.size(0),
                     out_rows, emb, out.data_ptr< T >());
   });
   return out;
}

// mp_ops.cpp:3103-3166 (loop 2838-2860, fallback 2930-2945)
Tensor fanout_scatter_backward_cpu(const Tensor& grad_out, const Tensor& src_global_idx, const Tensor& flat_dst,
                                   int64_t x_rows)
{
   check_rank(grad_out, 2, "grad_out");
   check_int64_index(src_global_idx, "src_global_idx");
   check_int64_index(flat_dst, "flat_dst");
   TORCH_CHECK(src_global_idx.size(0) == flat_dst.size(0), "src_global_idx and flat_dst must have equal length.");
   TORCH_CHECK(x_rows >= 0, "x_rows must be >= 0.");
   const int64_t emb = grad_out.size(1);
   Tensor grad_x = at::zeros({x_rows, emb}, grad_out.options());
   if(src_global_idx.numel() == 0 || x_rows == 0) return grad_x;
   if(!loop_dtype(grad_out)) {
      grad_x.index_add_(0, src_global_idx, grad_out.index_select(0, flat_dst));
      return grad_x;
   }
   const Tensor g = contig(grad_out), src = contig(src_global_idx), dst = contig(flat_dst);
   float_or_double(g, [&](auto v) {
      using T = decltype(v);
      add_rows< T >(g.data_ptr< T >(), dst.data_ptr< int64_t >(), g.size(0), "flat_dst", grad_x.data_ptr< T >(),
                    src.data_ptr< int64_t >(), x_rows, "src_global_idx", true, src.size(0), emb);
   });
   return grad_x;
}

// mp_ops.cpp:3168-3222 (loop 2862-2886, fallback 2947-2962)
Tensor fanin_reduce_sum_cpu(const Tensor& rel_flat, const Tensor& flat_src, const Tensor& dst_idx, int64_t dim_size)
{
   const int64_t emb = rel_flat.size(1);
   Tensor out = at::zeros({dim_size, emb}, rel_flat.options());
   if(flat_src.numel() == 0 || dim_size == 0) return out;
   if(!loop_dtype(rel_flat)) {
      out.index_add_(0, dst_idx, rel_flat.index_select(0, flat_src));
      return out;
   }
   const Tensor rel = contig(rel_flat), src = contig(flat_src), dst = contig(dst_idx);
   float_or_double(rel, [&](auto v) {
      using T = decltype(v);
      add_rows< T >(rel.data_ptr< T >(), src.data_ptr< int64_t >(), rel.size(0), "flat_src", out.data_ptr< T >(),
                    dst.data_ptr< int64_t >(), dim_size, "dst_idx", false, src.size(0), emb);
   });
   return out;
}

// The ATen formula of mp_ops.cpp:3005-3036: per column, the max over the row's
// messages, then log of the sum of exp(message - max), plus the max. Rows
// without messages stay -inf.
Tensor fanin_reduce_logsumexp_cpu(const Tensor& rel_flat, const Tensor& flat_src, const Tensor& dst_idx,
                                  int64_t dim_size)
{
   const int64_t emb = rel_flat.size(1);
   Tensor row_max = at::full({dim_size, emb}, -std::numeric_limits< double >::infinity(), rel_flat.options());
   if(flat_src.numel() == 0 || dim_size == 0) return row_max;
   const Tensor msgs = rel_flat.index_select(0, flat_src);
   const Tensor cols = dst_idx.unsqueeze(1).expand({dst_idx.size(0), emb});
   row_max.scatter_reduce_(0, cols, msgs, "amax", true);
   const Tensor shifted_exp = (msgs - row_max.index_select(0, dst_idx)).exp();
   Tensor sums = at::zeros({dim_size, emb}, rel_flat.options());
   sums.scatter_add_(0, cols, shifted_exp);
   return sums.log() + row_max;
}

// mp_ops.cpp:3327-3348
Tensor fanin_reduce_cpu(const Tensor& rel_flat, const Tensor& flat_src, const Tensor& dst_idx, int64_t dim_size,
                        int64_t mode)
{
   check_rank(rel_flat, 2, "rel_flat");
   check_int64_index(flat_src, "flat_src");
   check_int64_index(dst_idx, "dst_idx");
   TORCH_CHECK(flat_src.size(0) == dst_idx.size(0), "flat_src and dst_idx must have equal length.");
   TORCH_CHECK(dim_size >= 0, "dim_size must be >= 0.");
   if(mode == kModeSum) return fanin_reduce_sum_cpu(rel_flat, flat_src, dst_idx, dim_size);
   if(mode == kModeLogSumExp) return fanin_reduce_logsumexp_cpu(rel_flat, flat_src, dst_idx, dim_size);
   throw std::invalid_argument("Unsupported fanin_reduce mode. Supported: 0=sum, 1=logsumexp.");
}

// mp_ops.cpp:3224-3284 (loop 2888-2911, fallback 2964-2979)
Tensor fanin_reduce_sum_backward_cpu(const Tensor& grad_out, const Tensor& flat_src, const Tensor& dst_idx,
                                     int64_t rel_rows)
{
   check_rank(grad_out, 2, "grad_out");
   check_int64_index(flat_src, "flat_src");
   check_int64_index(dst_idx, "dst_idx");
   TORCH_CHECK(flat_src.size(0) == dst_idx.size(0), "flat_src and dst_idx must have equal length.");
   TORCH_CHECK(rel_rows >= 0, "rel_rows must be >= 0.");
   const int64_t emb = grad_out.size(1);
   Tensor grad_rel = at::zeros({rel_rows, emb}, grad_out.options());
   if(flat_src.numel() == 0 || rel_rows == 0) return grad_rel;
   if(!loop_dtype(grad_out)) {
      grad_rel.index_add_(0, flat_src, grad_out.index_select(0, dst_idx));
      return grad_rel;
   }
   const Tensor g = contig(grad_out), src = contig(flat_src), dst = contig(dst_idx);
   float_or_double(g, [&](auto v) {
      using T = decltype(v);
      add_rows< T >(g.data_ptr< T >(), dst.data_ptr< int64_t >(), g.size(0), "dst_idx", grad_rel.data_ptr< T >(),
                    src.data_ptr< int64_t >(), rel_rows, "flat_src", true, src.size(0), emb);
   });
   return grad_rel;
}

// mp_ops.cpp:3286-3325 with the ATen formula of 2981-3003:
// grad_rel[flat_src[e]] += grad_out[dst[e]] * exp(rel[flat_src[e]] - out[dst[e]]).
Tensor fanin_reduce_logsumexp_backward_cpu(const Tensor& grad_out, const Tensor& rel_flat, const Tensor& flat_src,
                                           const Tensor& dst_idx, const Tensor& out, int64_t rel_rows)
{
   check_rank(grad_out, 2, "grad_out");
   check_rank(rel_flat, 2, "rel_flat");
   check_int64_index(flat_src, "flat_src");
   check_int64_index(dst_idx, "dst_idx");
   check_rank(out, 2, "out");
   TORCH_CHECK(flat_src.size(0) == dst_idx.size(0), "flat_src and dst_idx must have equal length.");
   TORCH_CHECK(rel_flat.size(1) == grad_out.size(1), "rel_flat and grad_out must share embedding dim.");
   TORCH_CHECK(out.size(0) == grad_out.size(0), "out and grad_out must share dim_size.");
   TORCH_CHECK(out.size(1) == grad_out.size(1), "out and grad_out must share embedding dim.");
   TORCH_CHECK(rel_rows >= 0, "rel_rows must be >= 0.");
   const int64_t emb = grad_out.size(1);
   Tensor grad_rel = at::zeros({rel_rows, emb}, rel_flat.options());
   if(flat_src.numel() == 0 || rel_rows == 0) return grad_rel;
   const Tensor weight = (rel_flat.index_select(0, flat_src) - out.index_select(0, dst_idx)).exp();
   grad_rel.index_add_(0, flat_src, grad_out.index_select(0, dst_idx) * weight);
   return grad_rel;
}

// ---- smoothed logsumexp (relmo's LogSumExpAggregation, models/aggr.py:96-123) -------------
//
// The formula relmo's models evaluate for "logsumexp" aggregation: per column,
// m = row max over the messages (kept at 0 for rows without messages, no
// gradient), out = (1/beta) log(eps + sum e^(beta (x - m))) + m. Its backward
// weight is e^(beta (x - out)).

void check_smoothed(double beta, double eps)
{
   TORCH_CHECK(beta > 0.0 && std::isfinite(beta), "smoothed logsumexp needs a finite beta > 0.");
   TORCH_CHECK(eps >= 0.0, "smoothed logsumexp needs eps >= 0.");
}

Tensor smoothed_logsumexp_cpu(const Tensor& rel_flat, const Tensor& flat_src, const Tensor& dst_idx, int64_t dim_size,
                              double beta, double eps)
{
   check_rank(rel_flat, 2, "rel_flat");
   check_int64_index(flat_src, "flat_src");
   check_int64_index(dst_idx, "dst_idx");
   TORCH_CHECK(flat_src.size(0) == dst_idx.size(0), "flat_src and dst_idx must have equal length.");
   TORCH_CHECK(dim_size >= 0, "dim_size must be >= 0.");
   check_smoothed(beta, eps);
   const Tensor msgs = rel_flat.index_select(0, flat_src);
   Tensor row_max = at::zeros({dim_size, rel_flat.size(1)}, rel_flat.options());
   row_max.index_reduce_(0, dst_idx, msgs, "amax", /*include_self=*/false);
   Tensor sums = at::full_like(row_max, eps);
   sums.index_add_(0, dst_idx, (beta * (msgs - row_max.index_select(0, dst_idx))).exp());
   return (1.0 / beta) * sums.log() + row_max;
}

Tensor smoothed_logsumexp_backward_cpu(const Tensor& grad_out, const Tensor& rel_flat, const Tensor& flat_src,
                                       const Tensor& dst_idx, const Tensor& out, int64_t rel_rows, double beta)
{
   check_rank(grad_out, 2, "grad_out");
   check_rank(rel_flat, 2, "rel_flat");
   check_int64_index(flat_src, "flat_src");
   check_int64_index(dst_idx, "dst_idx");
   check_rank(out, 2, "out");
   TORCH_CHECK(flat_src.size(0) == dst_idx.size(0), "flat_src and dst_idx must have equal length.");
   TORCH_CHECK(rel_rows >= 0, "rel_rows must be >= 0.");
   check_smoothed(beta, 0.0);
   Tensor grad_rel = at::zeros({rel_rows, grad_out.size(1)}, rel_flat.options());
   if(flat_src.numel() == 0 || rel_rows == 0) return grad_rel;
   const Tensor weight = (beta * (rel_flat.index_select(0, flat_src) - out.index_select(0, dst_idx))).exp();
   grad_rel.index_add_(0, flat_src, grad_out.index_select(0, dst_idx) * weight);
   return grad_rel;
}

// ---- LGAN ops (sum / mean) --------------------------------------------------------

// One indexed aggregation (relmo/ops/mp_common.py:88-118, mp_ops.cpp:3433-3454):
// out[t] = sum of x[src[e]] over dst[e] = t, divided by max(count of t, 1) in
// mean mode.
Tensor lgan_agg(const Tensor& x, const Tensor& src, const Tensor& dst, int64_t rows, bool mean)
{
   Tensor out = x.new_zeros({rows, x.size(1)});
   if(src.numel() == 0 || dst.numel() == 0 || rows == 0) return out;
   out.index_add_(0, dst, x.index_select(0, src));
   if(!mean) return out;
   Tensor count = x.new_zeros({rows, 1});
   count.index_add_(0, dst, at::ones({dst.size(0), 1}, x.options()));
   return out / count.clamp_min_(1.0);
}

// Its reverse (mp_ops.cpp:3527-3555): g_src[s] = sum over src[e] = s of
// g[dst[e]] (divided by max(count of dst[e], 1) in mean mode).
Tensor lgan_agg_reverse(const Tensor& g, const Tensor& src, const Tensor& dst, int64_t rows, bool mean)
{
   Tensor out = g.new_zeros({rows, g.size(1)});
   if(src.numel() == 0 || dst.numel() == 0 || rows == 0) return out;
   Tensor picked = g.index_select(0, dst);
   if(mean) {
      Tensor count = g.new_zeros({g.size(0), 1});
      count.index_add_(0, dst, at::ones({dst.size(0), 1}, g.options()));
      picked = picked / count.index_select(0, dst).clamp_min_(1.0);
   }
   out.index_add_(0, src, picked);
   return out;
}

void check_lgan_index_types(const Tensor& rr_src, const Tensor& rr_dst, const Tensor& tn_rel, const Tensor& tn_ent,
                            const Tensor& nn_rel, const Tensor& nn_ent)
{
   check_int32_or_int64_index(rr_src, "rr_src");
   check_int32_or_int64_index(rr_dst, "rr_dst");
   check_int32_or_int64_index(tn_rel, "tn_rel");
   check_int32_or_int64_index(tn_ent, "tn_ent");
   check_int32_or_int64_index(nn_rel, "nn_rel");
   check_int32_or_int64_index(nn_ent, "nn_ent");
}

void check_one_device(const Tensor& ref, std::initializer_list< const Tensor* > ts, const char* op)
{
   bool same = true;
   for(const Tensor* t : ts) same = same && t->device() == ref.device();
   TORCH_CHECK(same, op, " expects all tensors on the same device.");
}

void check_lgan_mode(int64_t mode, const char* op)
{
   TORCH_CHECK(mode == kModeSum || mode == kModeMean, op, " supports only mode 0=sum or 2=mean.");
}

// mp_ops.cpp:3350-3469
std::tuple< Tensor, Tensor, Tensor > lgan_pool_reduce_cpu(const Tensor& slot_messages,
                                                          const Tensor& slot_to_relation_instance,
                                                          const Tensor& relation_instance_arities,
                                                          const Tensor& rr_src, const Tensor& rr_dst,
                                                          const Tensor& tn_rel, const Tensor& tn_ent,
                                                          const Tensor& nn_rel, const Tensor& nn_ent,
                                                          int64_t entity_dim_size, int64_t mode)
{
   check_rank(slot_messages, 2, "slot_messages");
   check_int32_or_int64_index(slot_to_relation_instance, "slot_to_relation_instance");
   check_int64_index(relation_instance_arities, "relation_instance_arities");
   check_lgan_index_types(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent);
   check_one_device(slot_messages, {&slot_to_relation_instance, &relation_instance_arities, &rr_src, &rr_dst, &tn_rel,
                                    &tn_ent, &nn_rel, &nn_ent},
                    "lgan_pool_reduce");
   TORCH_CHECK(entity_dim_size >= 0, "entity_dim_size must be >= 0.");
   TORCH_CHECK(slot_to_relation_instance.size(0) == slot_messages.size(0),
               "slot_to_relation_instance length must match slot_messages rows.");
   TORCH_CHECK(tn_rel.size(0) == tn_ent.size(0), "tn_rel and tn_ent must have equal length.");
   TORCH_CHECK(nn_rel.size(0) == nn_ent.size(0), "nn_rel and nn_ent must have equal length.");
   TORCH_CHECK(rr_src.size(0) == rr_dst.size(0), "rr_src and rr_dst must have equal length.");
   check_lgan_mode(mode, "lgan_pool_reduce");
   const bool mean = mode == kModeMean;
   const int64_t relations = relation_instance_arities.size(0);
   Tensor x = slot_messages.new_zeros({relations, slot_messages.size(1)});
   if(slot_messages.numel() > 0) {
      x.index_add_(0, slot_to_relation_instance, slot_messages);
      x = x / relation_instance_arities.to(slot_messages.scalar_type()).view({relations, 1}).clamp_min_(1.0);
   }
   x = x + lgan_agg(x, rr_src, rr_dst, relations, mean);
   Tensor tn = lgan_agg(x, tn_rel, tn_ent, entity_dim_size, mean);
   Tensor nn = lgan_agg(x, nn_rel, nn_ent, entity_dim_size, mean);
   return {x, tn, nn};
}

// mp_ops.cpp:3471-3572
Tensor lgan_pool_reduce_backward_cpu(const Tensor& grad_relation_pair_x, const Tensor& grad_tn_msgs,
                                     const Tensor& grad_nn_msgs, const Tensor& slot_to_relation_instance,
                                     const Tensor& relation_instance_arities, const Tensor& rr_src,
                                     const Tensor& rr_dst, const Tensor& tn_rel, const Tensor& tn_ent,
                                     const Tensor& nn_rel, const Tensor& nn_ent, int64_t relation_count, int64_t mode)
{
   check_rank(grad_relation_pair_x, 2, "grad_relation_pair_x");
   check_rank(grad_tn_msgs, 2, "grad_tn_msgs");
   check_rank(grad_nn_msgs, 2, "grad_nn_msgs");
   check_int32_or_int64_index(slot_to_relation_instance, "slot_to_relation_instance");
   check_int64_index(relation_instance_arities, "relation_instance_arities");
   check_lgan_index_types(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent);
   check_one_device(grad_relation_pair_x, {&grad_tn_msgs, &grad_nn_msgs, &slot_to_relation_instance,
                                           &relation_instance_arities, &rr_src, &rr_dst, &tn_rel, &tn_ent, &nn_rel,
                                           &nn_ent},
                    "lgan_pool_reduce_backward");
   check_lgan_mode(mode, "lgan_pool_reduce_backward");
   TORCH_CHECK(relation_count >= 0, "relation_count must be >= 0.");
   const bool mean = mode == kModeMean;
   Tensor g = grad_relation_pair_x.clone();
   g = g + lgan_agg_reverse(grad_tn_msgs, tn_rel, tn_ent, relation_count, mean) +
       lgan_agg_reverse(grad_nn_msgs, nn_rel, nn_ent, relation_count, mean);
   g = g + lgan_agg_reverse(g, rr_src, rr_dst, relation_count, mean);
   const int64_t slots = slot_to_relation_instance.size(0);
   const Tensor divisor = relation_instance_arities.to(g.scalar_type())
                             .index_select(0, slot_to_relation_instance.to(at::kLong))
                             .view({slots, 1})
                             .clamp_min_(1.0);
   return g.index_select(0, slot_to_relation_instance) / divisor;
}

// mp_ops.cpp:3574-3656
std::tuple< Tensor, Tensor, Tensor > lgan_relation_graph_step_cpu(const Tensor& relation_pair_x, const Tensor& rr_src,
                                                                  const Tensor& rr_dst, const Tensor& tn_rel,
                                                                  const Tensor& tn_ent, const Tensor& nn_rel,
                                                                  const Tensor& nn_ent, int64_t entity_dim_size,
                                                                  int64_t mode)
{
   check_rank(relation_pair_x, 2, "relation_pair_x");
   check_lgan_index_types(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent);
   check_one_device(relation_pair_x, {&rr_src, &rr_dst, &tn_rel, &tn_ent, &nn_rel, &nn_ent},
                    "lgan_relation_graph_step");
   TORCH_CHECK(entity_dim_size >= 0, "entity_dim_size must be >= 0.");
   TORCH_CHECK(rr_src.size(0) == rr_dst.size(0), "rr_src and rr_dst must have equal length.");
   TORCH_CHECK(tn_rel.size(0) == tn_ent.size(0), "tn_rel and tn_ent must have equal length.");
   TORCH_CHECK(nn_rel.size(0) == nn_ent.size(0), "nn_rel and nn_ent must have equal length.");
   check_lgan_mode(mode, "lgan_relation_graph_step");
   const bool mean = mode == kModeMean;
   Tensor x1 = relation_pair_x + lgan_agg(relation_pair_x, rr_src, rr_dst, relation_pair_x.size(0), mean);
   Tensor tn = lgan_agg(x1, tn_rel, tn_ent, entity_dim_size, mean);
   Tensor nn = lgan_agg(x1, nn_rel, nn_ent, entity_dim_size, mean);
   return {x1, tn, nn};
}

// mp_ops.cpp:3658-3743
Tensor lgan_relation_graph_step_backward_cpu(const Tensor& grad_relation_pair_x, const Tensor& grad_tn_msgs,
                                             const Tensor& grad_nn_msgs, const Tensor& rr_src, const Tensor& rr_dst,
                                             const Tensor& tn_rel, const Tensor& tn_ent, const Tensor& nn_rel,
                                             const Tensor& nn_ent, int64_t relation_count, int64_t mode)
{
   check_rank(grad_relation_pair_x, 2, "grad_relation_pair_x");
   check_rank(grad_tn_msgs, 2, "grad_tn_msgs");
   check_rank(grad_nn_msgs, 2, "grad_nn_msgs");
   check_lgan_index_types(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent);
   check_one_device(grad_relation_pair_x, {&grad_tn_msgs, &grad_nn_msgs, &rr_src, &rr_dst, &tn_rel, &tn_ent, &nn_rel,
                                           &nn_ent},
                    "lgan_relation_graph_step_backward");
   TORCH_CHECK(relation_count >= 0, "relation_count must be >= 0.");
   check_lgan_mode(mode, "lgan_relation_graph_step_backward");
   const bool mean = mode == kModeMean;
   Tensor g = grad_relation_pair_x + lgan_agg_reverse(grad_tn_msgs, tn_rel, tn_ent, relation_count, mean) +
              lgan_agg_reverse(grad_nn_msgs, nn_rel, nn_ent, relation_count, mean);
   return g + lgan_agg_reverse(g, rr_src, rr_dst, relation_count, mean);
}

}  // namespace
}  // namespace relm_b200

TORCH_LIBRARY_IMPL(relm_mp, CPU, m)
{
   m.impl("fanout_scatter", relm_b200::fanout_scatter_cpu);
   m.impl("fanout_scatter_backward", relm_b200::fanout_scatter_backward_cpu);
   m.impl("fanin_reduce", relm_b200::fanin_reduce_cpu);
   m.impl("fanin_reduce_sum_backward", relm_b200::fanin_reduce_sum_backward_cpu);
   m.impl("fanin_reduce_logsumexp_backward", relm_b200::fanin_reduce_logsumexp_backward_cpu);
   m.impl("lgan_pool_reduce", relm_b200::lgan_pool_reduce_cpu);
   m.impl("lgan_pool_reduce_backward", relm_b200::lgan_pool_reduce_backward_cpu);
   m.impl("lgan_relation_graph_step", relm_b200::lgan_relation_graph_step_cpu);
   m.impl("lgan_relation_graph_step_backward", relm_b200::lgan_relation_graph_step_backward_cpu);
}

TORCH_LIBRARY_IMPL(relm_mp_b200, CPU, m)
{
   m.impl("fanin_reduce_smoothed_logsumexp", relm_b200::smoothed_logsumexp_cpu);
   m.impl("fanin_reduce_smoothed_logsumexp_backward", relm_b200::smoothed_logsumexp_backward_cpu);
}
