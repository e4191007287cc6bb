// LGAN indexed reductions, `sum` and `mean` modes (relmo: src/_ops/mp/mp_ops.cpp
// 3350-3743 for the ops, src/relmo/ops/mp_common.py:88-118 for one indexed
// sum / mean). Every aggregation runs through a plan (CSR of the target index)
// and the planned sum with its fused epilogue (base + sum / divisor), so the
// mean division, the residual `x + rr_msgs` and the pool's division by the
// arities cost no pass of their own. The reverse aggregations of the backward
// ops are planned sums over the reversed index pair; in mean mode their
// gathered rows are first divided by the counts of the forward targets.
//
// The op-level entry points build their plans one at a time in the caller's
// workspace; the torch library calls the planned pieces with cached plans.
#include <cstdio>

#include "relm_mp_internal.cuh"

using namespace relm_mp;

namespace {

constexpr int kRowWarps = kThreads / 32;

__global__ void __launch_bounds__(kThreads) k_gather_counts(const int32_t* __restrict__ gidx, int64_t n,
                                                            int32_t* __restrict__ counts)
{
   const int64_t stride = (int64_t)gridDim.x * blockDim.x;
   for(int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += stride) atomicAdd(counts + gidx[j], 1);
}

__device__ __forceinline__ float load_acc(const float* p) { return *p; }
__device__ __forceinline__ double load_acc(const double* p) { return *p; }
__device__ __forceinline__ float load_acc(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load_acc(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ void store_acc(float* p, float v) { *p = v; }
__device__ __forceinline__ void store_acc(double* p, double v) { *p = v; }
__device__ __forceinline__ void store_acc(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void store_acc(__half* p, float v) { *p = __float2half_rn(v); }

// Warp per row, lanes over the columns (coalesced); grid-stride over rows.
template < typename T, typename A >
__global__ void __launch_bounds__(kThreads) k_divide_rows(const T* in, int64_t rows, int64_t emb,
                                                          const int32_t* __restrict__ counts, T* out)
{
   const int lane = threadIdx.x & 31;
   const int64_t nwarps = (int64_t)gridDim.x * kRowWarps;
   for(int64_t r = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5); r < rows; r += nwarps) {
      const int32_t c = counts[r];
      const A d = c > 1 ? (A)c : A(1);
      for(int64_t k = lane; k < emb; k += 32) store_acc(out + r * emb + k, load_acc(in + r * emb + k) / d);
   }
}

// 16-byte chunks (rows a multiple of 16 bytes, 16-byte aligned): thread per
// chunk, grid-stride; the divisor of a chunk's row comes from L1/L2.
template < typename T, typename A >
__global__ void __launch_bounds__(kThreads) k_divide_rows16(const T* in, int64_t chunks, int chunks_per_row,
                                                            const int32_t* __restrict__ counts, T* out)
{
   constexpr int VN = 16 / (int)sizeof(T);
   const int64_t stride = (int64_t)gridDim.x * blockDim.x;
   for(int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < chunks; c += stride) {
      const int32_t n = counts[c / chunks_per_row];
      const A d = n > 1 ? (A)n : A(1);
      uint4 v = *reinterpret_cast< const uint4* >(in + c * VN);
      T* e = reinterpret_cast< T* >(&v);
#pragma unroll
      for(int k = 0; k < VN; ++k) store_acc(e + k, load_acc(e + k) / d);
      *reinterpret_cast< uint4* >(out + c * VN) = v;
   }
}

// out[s] = table[index[s]] / max(div[index[s]], 1) (div may be null): thread
// per 16-byte chunk of an output row, grid-stride. The slots of one relation
// instance are adjacent, so a table row and its divisor are read from L1/L2
// after the first of them.
template < typename T, typename A >
__global__ void __launch_bounds__(kThreads) k_gather_div16(const T* __restrict__ table,
                                                           const int64_t* __restrict__ index, int64_t chunks,
                                                           int chunks_per_row, const int64_t* __restrict__ div,
                                                           T* __restrict__ out)
{
   const int64_t stride = (int64_t)gridDim.x * blockDim.x;
   for(int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < chunks; c += stride) {
      const int64_t s = c / chunks_per_row;
      const int64_t k = c - s * chunks_per_row;
      const int64_t g = __ldg(index + s);
      uint4 v = __ldg(reinterpret_cast< const uint4* >(table) + g * chunks_per_row + k);
      if(div) {
         const A dv = (A)__ldg(div + g);
         const A d = dv > A(1) ? dv : A(1);
         T* e = reinterpret_cast< T* >(&v);
#pragma unroll
         for(int i = 0; i < 16 / (int)sizeof(T); ++i) store_acc(e + i, load_acc(e + i) / d);
      }
      reinterpret_cast< uint4* >(out)[c] = v;
   }
}

// Element-wise form for rows that are not 16-byte multiples.
template < typename T, typename A >
__global__ void __launch_bounds__(kThreads) k_gather_div(const T* __restrict__ table, const int64_t* __restrict__ index,
                                                         int64_t n, int64_t emb, const int64_t* __restrict__ div,
                                                         T* __restrict__ out)
{
   const int64_t total = n * emb;
   const int64_t stride = (int64_t)gridDim.x * blockDim.x;
   for(int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
      const int64_t s = i / emb;
      const int64_t g = __ldg(index + s);
      A v = load_acc(table + g * emb + (i - s * emb));
      if(div) {
         const A dv = (A)__ldg(div + g);
         v = v / (dv > A(1) ? dv : A(1));
      }
      store_acc(out + i, v);
   }
}

template < typename T, typename A >
void launch_gather_div(const void* table, const int64_t* index, int64_t n, int64_t emb, const int64_t* div, void* out,
                       bool vec, cudaStream_t st);

unsigned grid_for(int64_t items, int64_t per_block, int64_t cap)
{
   int64_t b = (items + per_block - 1) / per_block;
   if(b > cap) b = cap;
   return (unsigned)(b < 1 ? 1 : b);
}

bool lgan_dtype_ok(relm_mp_dtype d)
{
   return d == RELM_MP_FLOAT32 || d == RELM_MP_FLOAT64 || d == RELM_MP_BFLOAT16 || d == RELM_MP_FLOAT16;
}

// One aggregation's plan plus scratch, carved from the op workspace.
struct AggMem {
   void* plan_mem;
   size_t plan_bytes;
   void* scratch;
   size_t scratch_bytes;
};

struct LganLayout {
   void* t1;         // [R, emb] values
   void* t2;         // [max(R, N), emb] values
   int32_t* counts;  // [max(R, N)]
   AggMem agg;
   size_t bytes;
};

size_t agg_bytes(int64_t edges, int64_t rows, int64_t emb, relm_mp_dtype dtype)
{
   return relm_mp_fanin_reduce_workspace_bytes(edges, rows, emb, dtype, RELM_MP_MODE_SUM);
}

LganLayout lgan_layout(void* ws, const relm_mp_lgan_graph& g, int64_t num_slots, int64_t emb, relm_mp_dtype dtype)
{
   const int64_t R = g.relation_count, N = g.entity_dim_size;
   const size_t es = dtype_size(dtype);
   const int64_t wide = R > N ? R : N;
   Carver c(ws);
   LganLayout l{};
   l.t1 = c.take< char >((size_t)R * (size_t)emb * es);
   l.t2 = c.take< char >((size_t)wide * (size_t)emb * es);
   l.counts = c.take< int32_t >((size_t)wide + 1);
   size_t agg = agg_bytes(num_slots, R, emb, dtype);
   // pool (slots -> R), rr (R -> R, both ways), tn / nn (R -> N forward, N -> R reverse)
   const size_t steps[5] = {
      agg_bytes(g.num_rr, R, emb, dtype), agg_bytes(g.num_tn, N, emb, dtype), agg_bytes(g.num_nn, N, emb, dtype),
      agg_bytes(g.num_tn, R, emb, dtype), agg_bytes(g.num_nn, R, emb, dtype)
   };
   for(size_t s : steps) agg = s > agg ? s : agg;
   char* rest = c.take< char >(agg);
   l.agg.plan_mem = rest;
   l.agg.plan_bytes = 0;
   l.agg.scratch = rest;
   l.agg.scratch_bytes = agg;
   l.bytes = c.used;
   return l;
}

struct Lgan {
   relm_mp_dtype dtype;
   const relm_mp_lgan_graph& g;
   int64_t emb;
   bool mean;
   LganLayout l;
   cudaStream_t st;

   // Builds the plan of (out_index, gather_index) in the aggregation memory.
   int plan(const int64_t* out_index, const int64_t* gather_index, int64_t edges, int64_t rows, int64_t gather_rows,
            const char* out_name, const char* gather_name, relm_mp_plan* p, AggMem* m)
   {
      const size_t pb = relm_mp_plan_bytes(edges, rows);
      m->plan_mem = l.agg.plan_mem;
      m->plan_bytes = pb;
      m->scratch = static_cast< char* >(l.agg.scratch) + pb;
      m->scratch_bytes = l.agg.scratch_bytes - pb;
      return relm_mp_plan_build_ex(
         out_index, gather_index, edges, rows, rows, gather_rows, out_name, gather_name, 0, m->plan_mem, pb,
         m->scratch, m->scratch_bytes, st, p
      );
   }

   // out[t] = base[t] + agg(table, src, dst)[t] (/ counts in mean mode; base may be null).
   int forward_agg(const void* table, int64_t table_rows, const int64_t* src, const int64_t* dst, int64_t edges,
                   int64_t rows, const char* src_name, const char* dst_name, const void* base, void* out)
   {
      relm_mp_plan p;
      AggMem m;
      int rc = plan(dst, src, edges, rows, table_rows, dst_name, src_name, &p, &m);
      if(rc) return rc;
      return relm_mp_plan_reduce_ex(&p, dtype, table, emb, base, nullptr, mean ? 1 : 0, out, m.scratch,
                                    m.scratch_bytes, st);
   }

   // out[s] = base[s] + sum over edges e with src[e] = s of grad[dst[e]] (/ count of dst[e] in mean mode):
   // the reverse of forward_agg.
   int reverse_agg(const void* grad, int64_t grad_rows, const int64_t* src, const int64_t* dst, int64_t edges,
                   int64_t rows, const char* src_name, const char* dst_name, const void* base, void* out)
   {
      relm_mp_plan p;
      AggMem m;
      int rc = plan(src, dst, edges, rows, grad_rows, src_name, dst_name, &p, &m);
      if(rc) return rc;
      const void* table = grad;
      if(mean && edges > 0 && grad_rows > 0 && emb > 0) {
         if((rc = relm_mp_plan_gather_counts(&p, l.counts, st))) return rc;
         if((rc = relm_mp_divide_rows(dtype, grad, grad_rows, emb, l.counts, l.t2, st))) return rc;
         table = l.t2;
      }
      return relm_mp_plan_reduce_ex(&p, dtype, table, emb, base, nullptr, 0, out, m.scratch, m.scratch_bytes, st);
   }

   int graph_forward(const void* x, void* x_out, void* tn, void* nn)
   {
      int rc = forward_agg(x, g.relation_count, g.rr_src, g.rr_dst, g.num_rr, g.relation_count, "rr_src", "rr_dst",
                           x, x_out);
      if(rc) return rc;
      rc = forward_agg(x_out, g.relation_count, g.tn_rel, g.tn_ent, g.num_tn, g.entity_dim_size, "tn_rel", "tn_ent",
                       nullptr, tn);
      if(rc) return rc;
      return forward_agg(x_out, g.relation_count, g.nn_rel, g.nn_ent, g.num_nn, g.entity_dim_size, "nn_rel",
                         "nn_ent", nullptr, nn);
   }

   // grad of the graph step's input into `out` (t1 holds the gradient of x1;
   // out may be t1 in mean mode only, where the rr table is t2).
   int graph_backward(const void* gx, const void* gtn, const void* gnn, void* out)
   {
      const int64_t R = g.relation_count, N = g.entity_dim_size;
      int rc = reverse_agg(gtn, N, g.tn_rel, g.tn_ent, g.num_tn, R, "tn_rel", "tn_ent", gx, l.t1);
      if(rc) return rc;
      if((rc = reverse_agg(gnn, N, g.nn_rel, g.nn_ent, g.num_nn, R, "nn_rel", "nn_ent", l.t1, l.t1))) return rc;
      return reverse_agg(l.t1, R, g.rr_src, g.rr_dst, g.num_rr, R, "rr_src", "rr_dst", l.t1, out);
   }
};

int check_lgan(relm_mp_dtype dtype, const relm_mp_lgan_graph* g, int64_t emb, int mode, const char* op)
{
   char msg[160];
   if(!g) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "graph must not be NULL.");
   if(!lgan_dtype_ok(dtype)) return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype.");
   if(mode != RELM_MP_MODE_SUM && mode != RELM_MP_MODE_MEAN) {
      snprintf(msg, sizeof msg, "%s supports only mode 0=sum or 2=mean.", op);
      return fail(RELM_MP_ERR_INVALID_ARGUMENT, msg);
   }
   if(emb < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "emb must be >= 0.");
   if(g->entity_dim_size < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "entity_dim_size must be >= 0.");
   if(g->relation_count < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "relation_count must be >= 0.");
   if(g->num_rr < 0 || g->num_tn < 0 || g->num_nn < 0)
      return fail(RELM_MP_ERR_INVALID_ARGUMENT, "edge counts must be >= 0.");
   return RELM_MP_OK;
}

int check_workspace(const LganLayout& l, void* ws, size_t ws_bytes)
{
   if(ws && ws_bytes >= l.bytes) return RELM_MP_OK;
   char msg[160];
   snprintf(msg, sizeof msg, "workspace too small: %zu bytes given, %zu needed.", ws_bytes, l.bytes);
   return fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, msg);
}

}  // namespace

int relm_mp_plan_gather_counts(const relm_mp_plan* plan, int32_t* counts, void* stream)
{
   if(!plan || !counts) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan and counts must not be NULL.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   if(plan->gather_rows == 0) return RELM_MP_OK;
   int rc = check_cuda(cudaMemsetAsync(counts, 0, (size_t)plan->gather_rows * sizeof(int32_t), st), "counts memset");
   if(rc || plan->num_edges == 0) return rc;
   k_gather_counts<<< grid_for(plan->num_edges, kThreads, 148 * 16), kThreads, 0, st >>>(
      plan->gidx, plan->num_edges, counts
   );
   return check_launch("k_gather_counts");
}

int relm_mp_divide_rows(relm_mp_dtype dtype, const void* in, int64_t rows, int64_t emb, const int32_t* counts,
                        void* out, void* stream)
{
   if(!lgan_dtype_ok(dtype)) return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype.");
   if(rows < 0 || emb < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "rows and emb must be >= 0.");
   if(rows == 0 || emb == 0) return RELM_MP_OK;
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   const int64_t row_bytes = emb * (int64_t)dtype_size(dtype);
   if(row_bytes % 16 == 0 && (reinterpret_cast< uintptr_t >(in) & 15u) == 0 &&
      (reinterpret_cast< uintptr_t >(out) & 15u) == 0) {
      const int cpr = (int)(row_bytes / 16);
      const int64_t chunks = rows * cpr;
      const unsigned g16 = grid_for(chunks, kThreads, 148 * 32);
      switch(dtype) {
         case RELM_MP_FLOAT32:
            k_divide_rows16< float, float ><<< g16, kThreads, 0, st >>>((const float*)in, chunks, cpr, counts,
                                                                         (float*)out);
            break;
         case RELM_MP_FLOAT64:
            k_divide_rows16< double, double ><<< g16, kThreads, 0, st >>>((const double*)in, chunks, cpr, counts,
                                                                           (double*)out);
            break;
         case RELM_MP_BFLOAT16:
            k_divide_rows16< __nv_bfloat16, float ><<< g16, kThreads, 0, st >>>(
               (const __nv_bfloat16*)in, chunks, cpr, counts, (__nv_bfloat16*)out
            );
            break;
         case RELM_MP_FLOAT16:
            k_divide_rows16< __half, float ><<< g16, kThreads, 0, st >>>((const __half*)in, chunks, cpr, counts,
                                                                          (__half*)out);
            break;
      }
      return check_launch("k_divide_rows16");
   }
   const unsigned grid = grid_for(rows, kRowWarps, 148 * 16);
   switch(dtype) {
      case RELM_MP_FLOAT32:
         k_divide_rows< float, float ><<< grid, kThreads, 0, st >>>((const float*)in, rows, emb, counts, (float*)out);
         break;
      case RELM_MP_FLOAT64:
         k_divide_rows< double, double ><<< grid, kThreads, 0, st >>>(
            (const double*)in, rows, emb, counts, (double*)out
         );
         break;
      case RELM_MP_BFLOAT16:
         k_divide_rows< __nv_bfloat16, float ><<< grid, kThreads, 0, st >>>(
            (const __nv_bfloat16*)in, rows, emb, counts, (__nv_bfloat16*)out
         );
         break;
      case RELM_MP_FLOAT16:
         k_divide_rows< __half, float ><<< grid, kThreads, 0, st >>>(
            (const __half*)in, rows, emb, counts, (__half*)out
         );
         break;
   }
   return check_launch("k_divide_rows");
}

namespace {

template < typename T, typename A >
void launch_gather_div(const void* table, const int64_t* index, int64_t n, int64_t emb, const int64_t* div, void* out,
                       bool vec, cudaStream_t st)
{
   if(vec) {
      const int cpr = (int)(emb * (int64_t)sizeof(T) / 16);
      const int64_t chunks = n * cpr;
      k_gather_div16< T, A ><<< grid_for(chunks, kThreads, 148 * 32), kThreads, 0, st >>>(
         static_cast< const T* >(table), index, chunks, cpr, div, static_cast< T* >(out)
      );
   } else {
      k_gather_div< T, A ><<< grid_for(n * emb, kThreads, 148 * 32), kThreads, 0, st >>>(
         static_cast< const T* >(table), index, n, emb, div, static_cast< T* >(out)
      );
   }
}

}  // namespace

int relm_mp_plan_gather_rows_div(const relm_mp_plan* plan, const int64_t* out_index, relm_mp_dtype dtype,
                                 const void* table, int64_t emb, const int64_t* row_div, void* out, void* stream)
{
   if(!plan) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan must not be NULL.");
   if(!lgan_dtype_ok(dtype)) return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype.");
   if(emb < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "emb must be >= 0.");
   if(plan->gather_rows != plan->num_edges)
      return fail(RELM_MP_ERR_INVALID_ARGUMENT, "the plan must gather the identity (one slot per edge).");
   const int64_t n = plan->num_edges;
   if(n == 0 || emb == 0) return RELM_MP_OK;
   if(!out_index || !table || !out) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "pointers must not be NULL.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   const size_t es = dtype_size(dtype);
   const bool vec = (emb * (int64_t)es) % 16 == 0 && (reinterpret_cast< uintptr_t >(table) & 15u) == 0 &&
                    (reinterpret_cast< uintptr_t >(out) & 15u) == 0;
   switch(dtype) {
      case RELM_MP_FLOAT32: launch_gather_div< float, float >(table, out_index, n, emb, row_div, out, vec, st); break;
      case RELM_MP_FLOAT64: launch_gather_div< double, double >(table, out_index, n, emb, row_div, out, vec, st); break;
      case RELM_MP_BFLOAT16:
         launch_gather_div< __nv_bfloat16, float >(table, out_index, n, emb, row_div, out, vec, st);
         break;
      case RELM_MP_FLOAT16: launch_gather_div< __half, float >(table, out_index, n, emb, row_div, out, vec, st); break;
   }
   return check_launch("k_gather_div");
}

size_t relm_mp_lgan_workspace_bytes(const relm_mp_lgan_graph* graph, int64_t num_slots, int64_t emb,
                                    relm_mp_dtype dtype)
{
   if(!graph || num_slots < 0 || emb < 0 || !lgan_dtype_ok(dtype)) return 0;
   return lgan_layout(nullptr, *graph, num_slots, emb, dtype).bytes;
}

// mp_ops.cpp:3574-3656
int relm_mp_lgan_relation_graph_step(relm_mp_dtype dtype, const relm_mp_lgan_graph* graph,
                                     const void* relation_pair_x, int64_t emb, int mode, void* relation_pair_x_out,
                                     void* tn_msgs, void* nn_msgs, void* workspace, size_t workspace_bytes,
                                     void* stream)
{
   int rc;
   if((rc = check_lgan(dtype, graph, emb, mode, "lgan_relation_graph_step"))) return rc;
   Lgan op{dtype, *graph, emb, mode == RELM_MP_MODE_MEAN, lgan_layout(workspace, *graph, 0, emb, dtype),
           static_cast< cudaStream_t >(stream)};
   if((rc = check_workspace(op.l, workspace, workspace_bytes))) return rc;
   return op.graph_forward(relation_pair_x, relation_pair_x_out, tn_msgs, nn_msgs);
}

// mp_ops.cpp:3658-3743
int relm_mp_lgan_relation_graph_step_backward(relm_mp_dtype dtype, const relm_mp_lgan_graph* graph,
                                              const void* grad_relation_pair_x, const void* grad_tn_msgs,
                                              const void* grad_nn_msgs, int64_t emb, int mode,
                                              void* grad_relation_pair_x_in, void* workspace,
                                              size_t workspace_bytes, void* stream)
{
   int rc;
   if((rc = check_lgan(dtype, graph, emb, mode, "lgan_relation_graph_step_backward"))) return rc;
   Lgan op{dtype, *graph, emb, mode == RELM_MP_MODE_MEAN, lgan_layout(workspace, *graph, 0, emb, dtype),
           static_cast< cudaStream_t >(stream)};
   if((rc = check_workspace(op.l, workspace, workspace_bytes))) return rc;
   return op.graph_backward(grad_relation_pair_x, grad_tn_msgs, grad_nn_msgs, grad_relation_pair_x_in);
}

// mp_ops.cpp:3350-3469
int relm_mp_lgan_pool_reduce(relm_mp_dtype dtype, const relm_mp_lgan_graph* graph, const void* slot_messages,
                             int64_t num_slots, int64_t emb, const int64_t* slot_to_relation_instance,
                             const int64_t* relation_instance_arities, int mode, void* relation_pair_x,
                             void* tn_msgs, void* nn_msgs, void* workspace, size_t workspace_bytes, void* stream)
{
   int rc;
   if((rc = check_lgan(dtype, graph, emb, mode, "lgan_pool_reduce"))) return rc;
   if(num_slots < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "num_slots must be >= 0.");
   Lgan op{dtype, *graph, emb, mode == RELM_MP_MODE_MEAN, lgan_layout(workspace, *graph, num_slots, emb, dtype),
           static_cast< cudaStream_t >(stream)};
   if((rc = check_workspace(op.l, workspace, workspace_bytes))) return rc;
   // x[r] = (sum of the slot rows of r) / max(arity[r], 1)
   relm_mp_plan p;
   AggMem m;
   if((rc = op.plan(slot_to_relation_instance, nullptr, num_slots, graph->relation_count, num_slots,
                    "slot_to_relation_instance", "slot", &p, &m)))
      return rc;
   if((rc = relm_mp_plan_reduce_ex(&p, dtype, slot_messages, emb, nullptr, relation_instance_arities, 0, op.l.t1,
                                   m.scratch, m.scratch_bytes, op.st)))
      return rc;
   return op.graph_forward(op.l.t1, relation_pair_x, tn_msgs, nn_msgs);
}

// mp_ops.cpp:3471-3572
int relm_mp_lgan_pool_reduce_backward(relm_mp_dtype dtype, const relm_mp_lgan_graph* graph,
                                      const void* grad_relation_pair_x, const void* grad_tn_msgs,
                                      const void* grad_nn_msgs, int64_t emb, int64_t num_slots,
                                      const int64_t* slot_to_relation_instance,
                                      const int64_t* relation_instance_arities, int mode, void* grad_slot_messages,
                                      void* workspace, size_t workspace_bytes, void* stream)
{
   int rc;
   if((rc = check_lgan(dtype, graph, emb, mode, "lgan_pool_reduce_backward"))) return rc;
   if(num_slots < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "num_slots must be >= 0.");
   const bool mean = mode == RELM_MP_MODE_MEAN;
   Lgan op{dtype, *graph, emb, mean, lgan_layout(workspace, *graph, num_slots, emb, dtype),
           static_cast< cudaStream_t >(stream)};
   if((rc = check_workspace(op.l, workspace, workspace_bytes))) return rc;
   // In sum mode the rr reverse gathers t1 itself, so its result goes to t2.
   void* grad_x = mean ? op.l.t1 : op.l.t2;
   if((rc = op.graph_backward(grad_relation_pair_x, grad_tn_msgs, grad_nn_msgs, grad_x))) return rc;
   // grad_slot[s] = grad_x[r] / max(arity[r], 1) for the relation r of slot s
   relm_mp_plan p;
   AggMem m;
   if((rc = op.plan(slot_to_relation_instance, nullptr, num_slots, graph->relation_count, num_slots,
                    "slot_to_relation_instance", "slot", &p, &m)))
      return rc;
   return relm_mp_plan_gather_rows_div(&p, slot_to_relation_instance, dtype, grad_x, emb, relation_instance_arities,
                                       grad_slot_messages, op.st);
}
