// C-ABI entry points of librelm_mp_b200.so (declared in include/relm_mp.h).
//
// Each op-level entry point reproduces one reference op of
// maichmueller/relmo src/_ops/mp/mp_ops.cpp (argument checks, early returns,
// output initialisation, error text) and runs it as:
//   plan build (relm_mp_plan.cu) -> one planned kernel (relm_mp_segment.cuh).
// The workspace holds the plan; the plan-build scratch and the reduction
// scratch share the space after it.
#include <atomic>
#include <cstdio>
#include <string>

#include "relm_mp_internal.cuh"
#include "relm_mp_segment.cuh"

#ifndef RELM_MP_KERNEL_CUDA_VERSION
#define RELM_MP_KERNEL_CUDA_VERSION "unknown"
#endif

namespace relm_mp {

namespace {
thread_local std::string g_last_error;
std::atomic< unsigned long long > g_launches{0};

__global__ void k_fill_f32(float* out, int64_t n, float v)
{
   for(int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
      out[i] = v;
}
__global__ void k_fill_f64(double* out, int64_t n, double v)
{
   for(int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
      out[i] = v;
}
__global__ void k_fill_u16(unsigned short* out, int64_t n, unsigned short v)
{
   for(int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
      out[i] = v;
}

bool aligned(const void* p, int bytes) { return ((uintptr_t)p % (uintptr_t)bytes) == 0; }

// Sets bit g of the cover bitmap for the gather row g of every edge; *dups = 1
// once a row is hit twice. One bit per row keeps the bitmap in L2 (2 MB for
// 2^24 rows), where the atomics resolve.
__global__ void k_cover(const int32_t* __restrict__ gidx, int64_t n, uint32_t* __restrict__ cover,
                        int32_t* __restrict__ dups)
{
   bool dup = false;
   for(int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x) {
      const uint32_t g = (uint32_t)gidx[j];
      const uint32_t bit = 1u << (g & 31u);
      dup |= (atomicOr(&cover[g >> 5], bit) & bit) != 0u;
   }
   if(__syncthreads_or(dup) && threadIdx.x == 0 && *((volatile int32_t*)dups) == 0) *dups = 1;
}

// Up to kPackParts index parts per launch, passed by value.
constexpr int kPackParts = 64;
struct PackParts {
   const int64_t* src[kPackParts];
   int64_t mul[kPackParts];
   int64_t add[kPackParts];
   int64_t start[kPackParts + 1];  // output position of each part; start[count] = end
   int count;
};

// out[o] = src_k[o - start_k] * mul_k + add_k for the part k holding o; a
// grid-stride walk over the launch's output range, the part found by binary
// search over the (<= 64) part starts.
__global__ void __launch_bounds__(kThreads) k_pack_index(const PackParts pk, int64_t* __restrict__ out)
{
   const int64_t lo = pk.start[0];
   const int64_t hi = pk.start[pk.count];
   for(int64_t o = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < hi; o += (int64_t)gridDim.x * blockDim.x) {
      int a = 0, b = pk.count - 1;  // last part with start <= o
      while(a < b) {
         const int m = (a + b + 1) >> 1;
         if(pk.start[m] <= o)
            a = m;
         else
            b = m - 1;
      }
      out[o] = __ldg(pk.src[a] + (o - pk.start[a])) * pk.mul[a] + pk.add[a];
   }
}

struct Shape {
   int vb;
   int chmax;
   int lanes;
   int ch;
   int col_blocks;
   int64_t block_cols;
};

Shape shape_for(int64_t emb, int es, int vb);

// One warp load moves one row: the narrowest vector width that still covers the
// row with <= 32 lanes, among the widths that divide the row size and every
// pointer's alignment. Rows wider than 32 x 16 bytes take several chunks per
// lane (the 16-byte or scalar width) and, past 4 chunks, several column blocks.
Shape choose_shape(int64_t emb, int es, const void* const* ptrs, int nptrs)
{
   const int64_t row_bytes = emb * es;
   auto valid = [&](int vb) {
      if(vb < es || row_bytes % vb != 0) return false;
      for(int i = 0; i < nptrs; ++i)
         if(ptrs[i] != nullptr && !aligned(ptrs[i], vb)) return false;
      return true;
   };
   int vb = 0;
   for(int w = es; w <= 16; w <<= 1) {
      if(valid(w) && row_bytes / w <= 32) {
         vb = w;
         break;
      }
   }
   if(vb == 0) vb = valid(16) ? 16 : es;  // wide row: several chunks per lane
   return shape_for(emb, es, vb);
}

// Row map and scatter: the packed shape (16-byte vectors, several rows per
// warp instruction) for rows of 16..256 bytes that are a power of two times 16
// with 16-byte aligned pointers, else one row per warp instruction.
Shape choose_map_shape(int64_t emb, int es, const void* const* ptrs, int nptrs)
{
   const int64_t row_bytes = emb * es;
   const int64_t lanes = row_bytes / 16;
   bool ok = row_bytes > 0 && row_bytes % 16 == 0 && lanes <= 16 && (lanes & (lanes - 1)) == 0;
   for(int i = 0; ok && i < nptrs; ++i) ok = ptrs[i] == nullptr || aligned(ptrs[i], 16);
   if(!ok) return choose_shape(emb, es, ptrs, nptrs);
   Shape s{};
   s.vb = 16;
   s.chmax = kPackedCh;
   s.lanes = (int)lanes;
   s.ch = 1;
   s.col_blocks = 1;
   s.block_cols = emb;
   return s;
}

// For the segment reduction: the widest vector width (16 bytes when the row
// size and pointers allow), lanes per row a power of two, so one load
// instruction moves 32 / lanes rows.
Shape choose_reduce_shape(int64_t emb, int es, const void* const* ptrs, int nptrs)
{
   const int64_t row_bytes = emb * es;
   int vb = 16;
   while(vb > es) {
      bool ok = row_bytes % vb == 0;
      for(int i = 0; ok && i < nptrs; ++i) ok = ptrs[i] == nullptr || aligned(ptrs[i], vb);
      if(ok) break;
      vb >>= 1;
   }
   if(vb < es) vb = es;
   if(row_bytes / vb > 32 && vb != 16) vb = es;  // chunked rows use the 16-byte or scalar width
   Shape s = shape_for(emb, es, vb);
   if(s.chmax == 1) {
      int l = 1;
      while(l < s.lanes) l <<= 1;
      s.lanes = l;
      s.block_cols = (int64_t)l * (vb / es);
   }
   return s;
}

// Shared-memory pipeline shape: rows of 16-byte multiples with 16-byte aligned
// tables, in column blocks of up to 1 KB; PB bytes per lane (4..32), B rows per
// stage of kStreamStageBytes. Returns pb = 0 when the row does not fit the pipeline.
struct StreamShape {
   int pb;
   int lanes;
   int rows_per_stage;
   int col_blocks;
   int64_t block_cols;  // elements
};

StreamShape choose_stream_shape(int64_t emb, int es, const void* const* ptrs, int nptrs)
{
   StreamShape s{};
   const int64_t row_bytes = emb * es;
   if(row_bytes <= 0 || row_bytes % 16 != 0) return s;
   for(int i = 0; i < nptrs; ++i)
      if(ptrs[i] != nullptr && !aligned(ptrs[i], 16)) return s;
   int64_t cbw;
   if(row_bytes <= 1024) {
      cbw = row_bytes;
      s.col_blocks = 1;
   } else if(row_bytes % 1024 == 0) {
      cbw = 1024;
      s.col_blocks = (int)(row_bytes / 1024);
   } else {
      return s;
   }
   int pb = 0;
   for(int w = 4; w <= 32; w <<= 1) {
      if(w >= es && 32 * w >= cbw && cbw % w == 0) {
         pb = w;
         break;
      }
   }
   if(pb == 0 || ((cbw / 16) & (cbw / 16 - 1)) != 0) return s;  // 16-byte chunks per row: a power of two
   s.pb = pb;
   s.lanes = (int)(cbw / pb);
   const int64_t rows = kStreamStageBytes / cbw;
   s.rows_per_stage = (int)(rows > 32 ? 32 : (rows < 1 ? 1 : rows));
   s.block_cols = cbw / es;
   return s;
}

Shape shape_for(int64_t emb, int es, int vb)
{
   Shape s{};
   const int64_t row_bytes = emb * es;
   s.vb = vb;
   const int vn = vb / es;
   const int64_t nvec = row_bytes / vb;
   if(nvec <= 32) {
      s.lanes = (int)(nvec < 1 ? 1 : nvec);
      s.chmax = 1;
      s.ch = 1;
      s.block_cols = (int64_t)32 * vn;
      s.col_blocks = 1;
   } else {
      s.lanes = 32;
      s.chmax = 4;
      const int64_t need = (nvec + 31) / 32;
      s.ch = need < 4 ? (int)need : 4;
      s.block_cols = (int64_t)32 * s.ch * vn;
      s.col_blocks = (int)((emb + s.block_cols - 1) / s.block_cols);
   }
   return s;
}

struct ReduceScratch {
   void* head_val;
   void* tail_val;
   void* head_aux;
   void* tail_aux;
   int32_t* head_row;
   int32_t* tail_row;
   int32_t* long_count;
   int32_t* long_list;
   int64_t max_long;
   size_t bytes;
};

// A long row spans more than kLongRowTiles tiles and neighbouring long rows
// share at most one tile, so there are at most num_tiles / kLongRowTiles + 1.
int64_t max_long_rows(int64_t num_tiles)
{
   return num_tiles / kLongRowTiles + 1;
}

ReduceScratch reduce_layout(void* mem, int64_t num_tiles, int64_t emb, int acc_bytes, int mode)
{
   Carver c(mem);
   ReduceScratch r{};
   const size_t vals = (size_t)num_tiles * (size_t)emb * (size_t)acc_bytes;
   r.head_val = c.take< char >(vals);
   r.tail_val = c.take< char >(vals);
   r.head_aux = mode == RELM_MP_MODE_LOGSUMEXP ? c.take< char >(vals) : nullptr;
   r.tail_aux = mode == RELM_MP_MODE_LOGSUMEXP ? c.take< char >(vals) : nullptr;
   r.head_row = c.take< int32_t >((size_t)num_tiles);
   r.tail_row = c.take< int32_t >((size_t)num_tiles);
   r.max_long = max_long_rows(num_tiles);
   r.long_count = c.take< int32_t >(1);
   r.long_list = c.take< int32_t >((size_t)r.max_long);
   r.bytes = c.used;
   return r;
}

int acc_bytes_of(relm_mp_dtype d) { return d == RELM_MP_FLOAT64 ? 8 : 4; }

bool valid_dtype(relm_mp_dtype d)
{
   return d == RELM_MP_FLOAT32 || d == RELM_MP_FLOAT64 || d == RELM_MP_BFLOAT16 || d == RELM_MP_FLOAT16;
}

// The plain logsumexp of fanin_reduce mode 1.
void set_plain_lse(SegParams& p)
{
   p.lse_k = kLog2E;
   p.lse_eps = 0.0;
   p.lse_inv_beta = 1.0;
   p.lse_empty = -INFINITY;
}

// Value of a row without messages in the smoothed form, (1/beta) log(eps),
// evaluated in the accumulator type as the reference does it in the tensor's
// (fp32 for fp32 / bf16 / fp16 tables).
double smoothed_empty(relm_mp_dtype dtype, const relm_mp_lse_form& f)
{
   if(dtype == RELM_MP_FLOAT64) return (1.0 / f.beta) * log(f.eps);
   const float inv = 1.0f / (float)f.beta;
   return (double)(inv * logf((float)f.eps));
}

// The smoothed logsumexp (relmo's LogSumExpAggregation), or the plain one
// for a NULL form.
int set_lse_form(SegParams& p, relm_mp_dtype dtype, const relm_mp_lse_form* f)
{
   set_plain_lse(p);
   if(!f) return RELM_MP_OK;
   if(!(f->beta > 0.0) || !(f->eps >= 0.0) || !isfinite(f->beta))
      return fail(RELM_MP_ERR_INVALID_ARGUMENT, "logsumexp form needs beta > 0 and eps >= 0.");
   p.lse_k = f->beta * kLog2E;
   p.lse_eps = f->eps;
   p.lse_inv_beta = dtype == RELM_MP_FLOAT64 ? 1.0 / f->beta : (double)(1.0f / (float)f->beta);
   p.lse_empty = smoothed_empty(dtype, *f);
   return RELM_MP_OK;
}

SegParams base_params(const relm_mp_plan* plan, int64_t emb, const Shape& s)
{
   SegParams p{};
   p.row_ptr = plan->row_ptr;
   p.gidx = plan->gidx;
   p.tile_row = plan->tile_row;
   p.tile_edge = plan->tile_edge;
   p.has_dups = plan->device_flags;
   p.num_tiles = plan->num_tiles;
   p.num_rows = plan->num_rows;
   p.num_edges = plan->num_edges;
   p.tile_items = plan->tile_items;
   p.emb = emb;
   p.lanes = s.lanes;
   p.ch = s.ch;
   p.col_blocks = s.col_blocks;
   p.block_cols = s.block_cols;
   set_plain_lse(p);
   return p;
}

int dispatch_gather(relm_mp_dtype dtype, const SegParams& p, const Shape& s, cudaStream_t st)
{
   switch(dtype) {
      case RELM_MP_FLOAT32: return launch_row_map< float >(p, kCopyLast, s.vb, s.chmax, st);
      case RELM_MP_FLOAT64: return launch_row_map< double >(p, kCopyLast, s.vb, s.chmax, st);
      case RELM_MP_BFLOAT16: return launch_row_map< __nv_bfloat16 >(p, kCopyLast, s.vb, s.chmax, st);
      case RELM_MP_FLOAT16: return launch_row_map< __half >(p, kCopyLast, s.vb, s.chmax, st);
   }
   return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype");
}

int dispatch_scatter(relm_mp_dtype dtype, const SegParams& p, const Shape& s, const uint32_t* cover, int64_t rows,
                     cudaStream_t st)
{
   switch(dtype) {
      case RELM_MP_FLOAT32: return launch_scatter_rows< float >(p, cover, rows, s.vb, s.chmax, st);
      case RELM_MP_FLOAT64: return launch_scatter_rows< double >(p, cover, rows, s.vb, s.chmax, st);
      case RELM_MP_BFLOAT16: return launch_scatter_rows< __nv_bfloat16 >(p, cover, rows, s.vb, s.chmax, st);
      case RELM_MP_FLOAT16: return launch_scatter_rows< __half >(p, cover, rows, s.vb, s.chmax, st);
   }
   return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype");
}

int dispatch_reduce(relm_mp_dtype dtype, const SegParams& pm, const Shape& sm, const SegParams& pr,
                    const Shape& sr, int mode, cudaStream_t st)
{
   switch(dtype) {
      case RELM_MP_FLOAT32: return launch_seg_reduce< float >(pm, sm.vb, sm.chmax, pr, sr.vb, sr.chmax, mode, st);
      case RELM_MP_FLOAT64: return launch_seg_reduce< double >(pm, sm.vb, sm.chmax, pr, sr.vb, sr.chmax, mode, st);
      case RELM_MP_BFLOAT16:
         return launch_seg_reduce< __nv_bfloat16 >(pm, sm.vb, sm.chmax, pr, sr.vb, sr.chmax, mode, st);
      case RELM_MP_FLOAT16: return launch_seg_reduce< __half >(pm, sm.vb, sm.chmax, pr, sr.vb, sr.chmax, mode, st);
   }
   return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype");
}

int dispatch_stream(relm_mp_dtype dtype, const SegParams& pm, const Shape& sm, const SegParams& pst, int pb, int mode,
                    cudaStream_t st)
{
   switch(dtype) {
      case RELM_MP_FLOAT32: return launch_seg_stream< float >(pm, sm.vb, sm.chmax, pst, pb, mode, st);
      case RELM_MP_FLOAT64: return launch_seg_stream< double >(pm, sm.vb, sm.chmax, pst, pb, mode, st);
      case RELM_MP_BFLOAT16: return launch_seg_stream< __nv_bfloat16 >(pm, sm.vb, sm.chmax, pst, pb, mode, st);
      case RELM_MP_FLOAT16: return launch_seg_stream< __half >(pm, sm.vb, sm.chmax, pst, pb, mode, st);
   }
   return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype");
}

// Epilogue of a planned sum (relm_mp_plan_reduce_ex): out = base + sum / divisor.
struct SumEpilogue {
   const void* base = nullptr;
   const int64_t* row_div = nullptr;
   int divide_by_count = 0;
   bool on() const { return base || row_div || divide_by_count; }
};

// Planned reduction shared by relm_mp_plan_reduce / relm_mp_plan_logsumexp_backward.
int planned_reduce(const relm_mp_plan* plan, relm_mp_dtype dtype, int seg_mode, const void* table,
                   const void* table2, const void* own, int64_t emb, void* out, void* scratch,
                   size_t scratch_bytes, cudaStream_t stream, const SumEpilogue& epi = SumEpilogue(),
                   const relm_mp_lse_form* form = nullptr)
{
   if(!plan) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan must not be NULL.");
   if(!valid_dtype(dtype)) return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype.");
   if(emb < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "emb must be >= 0.");
   const int64_t es = (int64_t)dtype_size(dtype);
   if(plan->num_rows == 0 || emb == 0) return RELM_MP_OK;
   const int scratch_mode = seg_mode == kLse ? RELM_MP_MODE_LOGSUMEXP : RELM_MP_MODE_SUM;
   const ReduceScratch rs = reduce_layout(scratch, plan->num_tiles, emb, acc_bytes_of(dtype), scratch_mode);
   if(!scratch || scratch_bytes < rs.bytes)
      return fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, "reduce scratch is smaller than relm_mp_plan_reduce_scratch_bytes().");
   if(plan->num_edges == 0) {
      if(epi.base) {  // base + 0 / d = base
         if(epi.base == out) return RELM_MP_OK;
         return check_cuda(
            cudaMemcpyAsync(out, epi.base, (size_t)(plan->num_rows * emb * es), cudaMemcpyDeviceToDevice, stream),
            "epilogue base copy"
         );
      }
      if(seg_mode != kLse) return fill_rows(dtype, out, plan->num_rows * emb, false, stream);
      SegParams f{};
      if(const int rc = set_lse_form(f, dtype, form)) return rc;
      return fill_value(dtype, out, plan->num_rows * emb, f.lse_empty, stream);
   }
   const void* ptrs[5] = {table, table2, own, out, epi.base};
   const Shape s = choose_map_shape(emb, (int)es, ptrs, 5);
   const Shape sr = choose_reduce_shape(emb, (int)es, ptrs, 5);
   SegParams p = base_params(plan, emb, s);
   if(const int rc = set_lse_form(p, dtype, form)) return rc;
   p.table = table;
   p.table2 = table2;
   p.own = own;
   p.out = out;
   p.head_val = rs.head_val;
   p.tail_val = rs.tail_val;
   p.head_aux = rs.head_aux;
   p.tail_aux = rs.tail_aux;
   p.head_row = rs.head_row;
   p.tail_row = rs.tail_row;
   p.long_count = rs.long_count;
   p.long_list = rs.long_list;
   p.max_long = rs.max_long;
   // rows of 16..256 bytes (packed): plans without long rows go to the short-row kernel
   p.short_rows = s.chmax == kPackedCh ? 1 : 0;
   p.launch = kLaunchAll;
   if(plan->flags & RELM_MP_PLAN_FLAGS_KNOWN) {  // launch only the family the plan needs
      if(!(plan->flags & RELM_MP_PLAN_REPEATS))
         p.launch = kLaunchRowMap;
      else if(p.short_rows && !(plan->flags & RELM_MP_PLAN_LONG_ROWS))
         p.launch = kLaunchShort;
      else
         p.launch = kLaunchMerge;
   }
   if(seg_mode == kSum && epi.on()) {
      seg_mode = kSumEpi;
      p.epi_base = epi.base;
      p.epi_div = epi.row_div;
      p.epi_count = epi.divide_by_count ? 1 : 0;
   }
   int rc = (p.launch & kLaunchMerge)
               ? check_cuda(cudaMemsetAsync(rs.long_count, 0, sizeof(int32_t), stream), "long_count memset")
               : RELM_MP_OK;
   if(rc) return rc;
   const StreamShape ss = choose_stream_shape(emb, (int)es, ptrs, 5);
   if(ss.pb > 0) {
      SegParams pst = p;
      pst.lanes = ss.lanes;
      pst.ch = ss.rows_per_stage;
      pst.col_blocks = ss.col_blocks;
      pst.block_cols = ss.block_cols;
      return dispatch_stream(dtype, p, s, pst, ss.pb, seg_mode, stream);
   }
   SegParams pr = p;
   pr.lanes = sr.lanes;
   pr.ch = sr.ch;
   pr.col_blocks = sr.col_blocks;
   pr.block_cols = sr.block_cols;
   return dispatch_reduce(dtype, p, s, pr, sr, seg_mode, stream);
}

}  // namespace

int fail(int status, const std::string& message)
{
   g_last_error = message;
   return status;
}

int check_cuda(cudaError_t err, const char* what)
{
   if(err == cudaSuccess) return RELM_MP_OK;
   return fail(RELM_MP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

int check_launch(const char* what)
{
   g_launches.fetch_add(1, std::memory_order_relaxed);
   return check_cuda(cudaGetLastError(), what);
}

size_t dtype_size(relm_mp_dtype dtype)
{
   switch(dtype) {
      case RELM_MP_FLOAT32: return 4;
      case RELM_MP_FLOAT64: return 8;
      case RELM_MP_BFLOAT16: return 2;
      case RELM_MP_FLOAT16: return 2;
   }
   return 0;
}

int fill_rows(relm_mp_dtype dtype, void* out, int64_t count, bool neg_inf, cudaStream_t stream)
{
   if(count <= 0) return RELM_MP_OK;
   if(!neg_inf) return check_cuda(cudaMemsetAsync(out, 0, (size_t)count * dtype_size(dtype), stream), "zero fill");
   return fill_value(dtype, out, count, -INFINITY, stream);
}

int fill_value(relm_mp_dtype dtype, void* out, int64_t count, double value, cudaStream_t stream)
{
   if(count <= 0) return RELM_MP_OK;
   int64_t blocks = (count + kThreads - 1) / kThreads;
   if(blocks > 148 * 32) blocks = 148 * 32;
   switch(dtype) {
      case RELM_MP_FLOAT32: k_fill_f32<<< (unsigned)blocks, kThreads, 0, stream >>>((float*)out, count, (float)value); break;
      case RELM_MP_FLOAT64: k_fill_f64<<< (unsigned)blocks, kThreads, 0, stream >>>((double*)out, count, value); break;
      case RELM_MP_BFLOAT16: {
         const __nv_bfloat16 h = __float2bfloat16_rn((float)value);
         k_fill_u16<<< (unsigned)blocks, kThreads, 0, stream >>>((unsigned short*)out, count,
                                                                   *reinterpret_cast< const unsigned short* >(&h));
         break;
      }
      case RELM_MP_FLOAT16: {
         const __half h = __float2half_rn((float)value);
         k_fill_u16<<< (unsigned)blocks, kThreads, 0, stream >>>((unsigned short*)out, count,
                                                                   *reinterpret_cast< const unsigned short* >(&h));
         break;
      }
   }
   return check_launch("fill");
}

}  // namespace relm_mp

using namespace relm_mp;

namespace {

// Workspace of one op call: the plan, then the larger of the plan-build scratch
// and the reduction scratch (they are never live at the same time).
size_t op_workspace(int64_t num_edges, int64_t num_rows, int64_t emb, relm_mp_dtype dtype, int scratch_mode,
                    bool reduces)
{
   if(num_edges < 0 || num_rows < 0 || emb < 0) return 0;
   const size_t plan = relm_mp_plan_bytes(num_edges, num_rows);
   size_t scratch = relm_mp_plan_scratch_bytes(num_edges, num_rows);
   if(reduces) {
      const int64_t tiles = plan_num_tiles(num_edges, num_rows);
      const size_t red = reduce_layout(nullptr, tiles, emb, acc_bytes_of(dtype), scratch_mode).bytes;
      if(red > scratch) scratch = red;
   }
   return plan + scratch;
}

struct OpMem {
   void* plan_mem;
   size_t plan_bytes;
   void* scratch;
   size_t scratch_bytes;
};

int split_workspace(void* ws, size_t ws_bytes, size_t need, int64_t num_edges, int64_t num_rows, OpMem& m)
{
   if(!ws || ws_bytes < need) {
      char msg[160];
      snprintf(msg, sizeof msg, "workspace too small: %zu bytes given, %zu needed.", ws_bytes, need);
      return fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, msg);
   }
   m.plan_mem = ws;
   m.plan_bytes = relm_mp_plan_bytes(num_edges, num_rows);
   m.scratch = static_cast< char* >(ws) + m.plan_bytes;
   m.scratch_bytes = ws_bytes - m.plan_bytes;
   return RELM_MP_OK;
}

int check_common(relm_mp_dtype dtype, int64_t emb, int64_t num_edges)
{
   if(!valid_dtype(dtype)) return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype.");
   if(emb < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "emb must be >= 0.");
   if(num_edges < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "num_edges must be >= 0.");
   return RELM_MP_OK;
}

}  // namespace

extern "C" {

const char* relm_mp_status_string(int status)
{
   switch(status) {
      case RELM_MP_OK: return "RELM_MP_OK";
      case RELM_MP_ERR_INVALID_ARGUMENT: return "RELM_MP_ERR_INVALID_ARGUMENT";
      case RELM_MP_ERR_INDEX_OUT_OF_RANGE: return "RELM_MP_ERR_INDEX_OUT_OF_RANGE";
      case RELM_MP_ERR_WORKSPACE_TOO_SMALL: return "RELM_MP_ERR_WORKSPACE_TOO_SMALL";
      case RELM_MP_ERR_UNSUPPORTED: return "RELM_MP_ERR_UNSUPPORTED";
      case RELM_MP_ERR_CUDA: return "RELM_MP_ERR_CUDA";
   }
   return "RELM_MP_ERR_UNKNOWN";
}

const char* relm_mp_build_info(void)
{
   return "lib=relm_mp_b200;arch=sm_100a;kernel_cuda=" RELM_MP_KERNEL_CUDA_VERSION ";abi=1";
}

const char* relm_mp_last_error(void) { return g_last_error.c_str(); }

unsigned long long relm_mp_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

size_t relm_mp_plan_reduce_scratch_bytes(const relm_mp_plan* plan, int64_t emb, relm_mp_dtype dtype, int mode)
{
   if(!plan || emb < 0) return 0;
   return reduce_layout(nullptr, plan->num_tiles, emb, acc_bytes_of(dtype), mode).bytes;
}

int relm_mp_plan_gather_last(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* table, int64_t emb,
                             void* out, void* stream)
{
   if(!plan) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan must not be NULL.");
   if(!valid_dtype(dtype)) return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype.");
   if(emb < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "emb must be >= 0.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   if(plan->num_rows == 0 || emb == 0) return RELM_MP_OK;
   if(plan->num_edges == 0) return fill_rows(dtype, out, plan->num_rows * emb, false, st);
   const void* ptrs[2] = {table, out};
   const Shape s = choose_map_shape(emb, (int)dtype_size(dtype), ptrs, 2);
   SegParams p = base_params(plan, emb, s);
   p.table = table;
   p.out = out;
   return dispatch_gather(dtype, p, s, st);
}

int relm_mp_pack_index(const relm_mp_index_part* parts, int num_parts, int64_t* out, void* stream)
{
   if(num_parts < 0 || (num_parts > 0 && !parts)) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "parts must not be NULL.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   int64_t start = 0;
   PackParts pk{};
   auto flush = [&]() -> int {
      if(pk.count == 0) return RELM_MP_OK;
      const int64_t total = pk.start[pk.count];
      int64_t blocks = (total - pk.start[0] + kThreads - 1) / kThreads;
      if(blocks > 148 * 16) blocks = 148 * 16;
      k_pack_index<<< (unsigned)blocks, kThreads, 0, st >>>(pk, out);
      pk.count = 0;
      return check_launch("k_pack_index");
   };
   for(int k = 0; k < num_parts; ++k) {
      const relm_mp_index_part& q = parts[k];
      if(q.len < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "part lengths must be >= 0.");
      if(q.len == 0) continue;
      if(!q.src || !out) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "index pointers must not be NULL.");
      pk.src[pk.count] = q.src;
      pk.mul[pk.count] = q.mul;
      pk.add[pk.count] = q.add;
      pk.start[pk.count] = start;
      start += q.len;
      pk.start[pk.count + 1] = start;
      if(++pk.count == kPackParts) {
         const int rc = flush();
         if(rc) return rc;
      }
   }
   return flush();
}

int relm_mp_plan_gather_cover(const relm_mp_plan* plan, uint32_t* cover, int* has_dups, void* stream)
{
   if(!plan || !cover || !has_dups) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan, cover and has_dups must not be NULL.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   int rc;
   // The last int of the cover buffer's allocation is not ours: keep the flag
   // in the plan's own spare device flags word (index 3; words 0-2 hold the
   // plan's row facts, which later reductions read), cleared first.
   int32_t* flag = const_cast< int32_t* >(plan->device_flags) + 3;
   if((rc = check_cuda(cudaMemsetAsync(cover, 0, relm_mp_cover_words(plan->gather_rows) * sizeof(uint32_t), st),
                       "cover memset")))
      return rc;
   if((rc = check_cuda(cudaMemsetAsync(flag, 0, sizeof(int32_t), st), "cover flag memset"))) return rc;
   if(plan->num_edges > 0) {
      int64_t blocks = (plan->num_edges + kThreads - 1) / kThreads;
      if(blocks > 148 * 16) blocks = 148 * 16;
      k_cover<<< (unsigned)blocks, kThreads, 0, st >>>(plan->gidx, plan->num_edges, cover, flag);
      if((rc = check_launch("k_cover"))) return rc;
   }
   int32_t host = 0;
   if((rc = check_cuda(cudaMemcpyAsync(&host, flag, sizeof(int32_t), cudaMemcpyDeviceToHost, st), "cover flag copy")))
      return rc;
   if((rc = check_cuda(cudaStreamSynchronize(st), "cover sync"))) return rc;
   *has_dups = host != 0;
   return RELM_MP_OK;
}

int relm_mp_plan_nonempty_rows(const relm_mp_plan* plan, int64_t* rows, void* stream)
{
   if(!plan || !rows) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan and rows must not be NULL.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   int rc;
   int32_t host = 0;
   if((rc = check_cuda(cudaMemcpyAsync(&host, plan->device_flags + 2, sizeof(int32_t), cudaMemcpyDeviceToHost, st),
                       "row count copy")))
      return rc;
   if((rc = check_cuda(cudaStreamSynchronize(st), "row count sync"))) return rc;
   *rows = host;
   return RELM_MP_OK;
}

namespace {

int scatter_rows(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* table, int64_t emb,
                 const int64_t* row_div, const uint32_t* cover, void* out, cudaStream_t st)
{
   if(!valid_dtype(dtype)) return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype.");
   if(emb < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "emb must be >= 0.");
   if(plan->gather_rows == 0 || emb == 0) return RELM_MP_OK;
   if(plan->num_edges == 0) return fill_rows(dtype, out, plan->gather_rows * emb, false, st);
   const void* ptrs[2] = {table, out};
   const Shape s = choose_map_shape(emb, (int)dtype_size(dtype), ptrs, 2);
   SegParams p = base_params(plan, emb, s);
   p.table = table;
   p.out = out;
   p.epi_div = row_div;
   return dispatch_scatter(dtype, p, s, cover, plan->gather_rows, st);
}

}  // namespace

int relm_mp_plan_scatter_rows(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* table, int64_t emb,
                              const uint32_t* cover, void* out, void* stream)
{
   if(!plan) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan must not be NULL.");
   return scatter_rows(plan, dtype, table, emb, nullptr, cover, out, static_cast< cudaStream_t >(stream));
}

int relm_mp_plan_scatter_rows_div(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* table, int64_t emb,
                                  const int64_t* row_div, const uint32_t* cover, void* out, void* stream)
{
   if(!plan) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan must not be NULL.");
   return scatter_rows(plan, dtype, table, emb, row_div, cover, out, static_cast< cudaStream_t >(stream));
}

int relm_mp_plan_scatter_logsumexp_backward(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* grad_out,
                                            const void* lse_out, const void* rel, int64_t emb, const uint32_t* cover,
                                            void* grad_rel, void* stream)
{
   return relm_mp_plan_scatter_logsumexp_backward_ex(plan, dtype, nullptr, grad_out, lse_out, rel, emb, cover,
                                                     grad_rel, stream);
}

int relm_mp_plan_scatter_logsumexp_backward_ex(const relm_mp_plan* plan, relm_mp_dtype dtype,
                                               const relm_mp_lse_form* form, const void* grad_out,
                                               const void* lse_out, const void* rel, int64_t emb,
                                               const uint32_t* cover, void* grad_rel, void* stream)
{
   if(!plan) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan must not be NULL.");
   if(!valid_dtype(dtype)) return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype.");
   if(emb < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "emb must be >= 0.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   if(plan->gather_rows == 0 || emb == 0) return RELM_MP_OK;
   if(plan->num_edges == 0) return fill_rows(dtype, grad_rel, plan->gather_rows * emb, false, st);
   const void* ptrs[4] = {grad_out, lse_out, rel, grad_rel};
   const Shape s = choose_map_shape(emb, (int)dtype_size(dtype), ptrs, 4);
   if(s.chmax != kPackedCh)
      return fail(RELM_MP_ERR_UNSUPPORTED, "destination-ordered logsumexp backward needs rows of 16..256 bytes "
                                           "(a power of two times 16) with 16-byte aligned tables.");
   SegParams p = base_params(plan, emb, s);
   if(const int rc = set_lse_form(p, dtype, form)) return rc;
   p.table = grad_out;
   p.table2 = lse_out;
   p.own = rel;
   p.out = grad_rel;
   switch(dtype) {
      case RELM_MP_FLOAT32: return launch_scatter_lse_bwd< float >(p, cover, plan->gather_rows, st);
      case RELM_MP_FLOAT64: return launch_scatter_lse_bwd< double >(p, cover, plan->gather_rows, st);
      case RELM_MP_BFLOAT16: return launch_scatter_lse_bwd< __nv_bfloat16 >(p, cover, plan->gather_rows, st);
      case RELM_MP_FLOAT16: return launch_scatter_lse_bwd< __half >(p, cover, plan->gather_rows, st);
   }
   return fail(RELM_MP_ERR_UNSUPPORTED, "unsupported dtype");
}

int relm_mp_plan_read_flags(relm_mp_plan* plan, void* stream)
{
   if(!plan || !plan->device_flags) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan must not be NULL.");
   int32_t f[2] = {0, 0};
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   int rc = check_cuda(cudaMemcpyAsync(f, plan->device_flags, sizeof f, cudaMemcpyDeviceToHost, st), "flags copy");
   if(rc || (rc = check_cuda(cudaStreamSynchronize(st), "flags sync"))) return rc;
   plan->flags |= RELM_MP_PLAN_FLAGS_KNOWN | (f[0] ? RELM_MP_PLAN_REPEATS : 0u) | (f[1] ? RELM_MP_PLAN_LONG_ROWS : 0u);
   return RELM_MP_OK;
}

int relm_mp_plan_reduce(const relm_mp_plan* plan, relm_mp_dtype dtype, int mode, const void* table, int64_t emb,
                        void* out, void* scratch, size_t scratch_bytes, void* stream)
{
   if(mode != RELM_MP_MODE_SUM && mode != RELM_MP_MODE_LOGSUMEXP)
      return fail(RELM_MP_ERR_INVALID_ARGUMENT, "Unsupported fanin_reduce mode. Supported: 0=sum, 1=logsumexp.");
   return planned_reduce(
      plan, dtype, mode == RELM_MP_MODE_SUM ? kSum : kLse, table, nullptr, nullptr, emb, out, scratch,
      scratch_bytes, static_cast< cudaStream_t >(stream)
   );
}

int relm_mp_plan_reduce_ex(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* table, int64_t emb,
                           const void* base, const int64_t* row_div, int divide_by_count, void* out,
                           void* scratch, size_t scratch_bytes, void* stream)
{
   SumEpilogue e;
   e.base = base;
   e.row_div = row_div;
   e.divide_by_count = divide_by_count;
   return planned_reduce(
      plan, dtype, kSum, table, nullptr, nullptr, emb, out, scratch, scratch_bytes,
      static_cast< cudaStream_t >(stream), e
   );
}

int relm_mp_plan_logsumexp_backward(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* grad_out,
                                    const void* lse_out, const void* rel, int64_t emb, void* grad_rel,
                                    void* scratch, size_t scratch_bytes, void* stream)
{
   return planned_reduce(
      plan, dtype, kLseBwd, grad_out, lse_out, rel, emb, grad_rel, scratch, scratch_bytes,
      static_cast< cudaStream_t >(stream)
   );
}

int relm_mp_plan_reduce_lse(const relm_mp_plan* plan, relm_mp_dtype dtype, const relm_mp_lse_form* form,
                            const void* table, int64_t emb, void* out, void* scratch, size_t scratch_bytes,
                            void* stream)
{
   return planned_reduce(
      plan, dtype, kLse, table, nullptr, nullptr, emb, out, scratch, scratch_bytes,
      static_cast< cudaStream_t >(stream), SumEpilogue(), form
   );
}

int relm_mp_plan_logsumexp_backward_ex(const relm_mp_plan* plan, relm_mp_dtype dtype, const relm_mp_lse_form* form,
                                       const void* grad_out, const void* lse_out, const void* rel, int64_t emb,
                                       void* grad_rel, void* scratch, size_t scratch_bytes, void* stream)
{
   return planned_reduce(
      plan, dtype, kLseBwd, grad_out, lse_out, rel, emb, grad_rel, scratch, scratch_bytes,
      static_cast< cudaStream_t >(stream), SumEpilogue(), form
   );
}

// ---- fanout_scatter (mp_ops.cpp:3038-3101) ---------------------------------

// fanout_scatter runs through the source plan (rows = x rows, gather index =
// flat_dst) when flat_dst covers every slot at most once; otherwise (repeated
// slots, last writer wins) through the slot plan. Workspace: source plan,
// cover counts, then the larger of the source plan's build scratch and the
// slot plan with its build scratch.
size_t fanout_workspace(int64_t num_edges, int64_t x_rows, int64_t out_rows)
{
   if(num_edges < 0 || x_rows < 0 || out_rows < 0) return 0;
   const size_t src_plan = relm_mp_plan_bytes(num_edges, x_rows);
   const size_t cover = align_up(relm_mp_cover_words(out_rows) * sizeof(uint32_t));
   const size_t a = relm_mp_plan_scratch_bytes(num_edges, x_rows);
   const size_t b = relm_mp_plan_bytes(num_edges, out_rows) + relm_mp_plan_scratch_bytes(num_edges, out_rows);
   return src_plan + cover + (a > b ? a : b);
}

size_t relm_mp_fanout_scatter_workspace_bytes(int64_t num_edges, int64_t x_rows, int64_t out_rows, int64_t emb,
                                              relm_mp_dtype dtype)
{
   (void)emb;
   (void)dtype;
   return fanout_workspace(num_edges, x_rows, out_rows);
}

int relm_mp_fanout_scatter(relm_mp_dtype dtype, const void* x_cat, int64_t x_rows, int64_t emb,
                           const int64_t* src_global_idx, const int64_t* flat_dst, int64_t num_edges,
                           int64_t out_rows, void* out, void* workspace, size_t workspace_bytes, void* stream)
{
   int rc;
   if((rc = check_common(dtype, emb, num_edges))) return rc;
   if(out_rows < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "out_rows must be >= 0.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   if(num_edges == 0 || out_rows == 0) return fill_rows(dtype, out, out_rows * emb, false, st);
   if(x_rows < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "x_rows must be >= 0.");
   const size_t need = fanout_workspace(num_edges, x_rows, out_rows);
   if(!workspace || workspace_bytes < need) {
      char msg[160];
      snprintf(msg, sizeof msg, "workspace too small: %zu bytes given, %zu needed.", workspace_bytes, need);
      return fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, msg);
   }
   char* ws = static_cast< char* >(workspace);
   const size_t src_plan_bytes = relm_mp_plan_bytes(num_edges, x_rows);
   uint32_t* cover = reinterpret_cast< uint32_t* >(ws + src_plan_bytes);
   char* rest = ws + src_plan_bytes + align_up((size_t)out_rows * sizeof(int32_t));
   const size_t rest_bytes = workspace_bytes - (size_t)(rest - ws);
   relm_mp_plan plan;
   // The reference loop checks src_global_idx before flat_dst at each edge.
   if((rc = plan_build_bounded(
          src_global_idx, flat_dst, num_edges, x_rows, x_rows, out_rows, "src_global_idx", "flat_dst", false, ws,
          src_plan_bytes, rest, rest_bytes, st, &plan
       )))
      return rc;
   int dups = 0;
   if((rc = relm_mp_plan_gather_cover(&plan, cover, &dups, stream))) return rc;
   if(!dups) return relm_mp_plan_scatter_rows(&plan, dtype, x_cat, emb, cover, out, stream);
   relm_mp_plan slot_plan;
   const size_t slot_bytes = relm_mp_plan_bytes(num_edges, out_rows);
   if((rc = plan_build_bounded(
          flat_dst, src_global_idx, num_edges, out_rows, out_rows, x_rows, "flat_dst", "src_global_idx", true, rest,
          slot_bytes, rest + slot_bytes, rest_bytes - slot_bytes, st, &slot_plan
       )))
      return rc;
   return relm_mp_plan_gather_last(&slot_plan, dtype, x_cat, emb, out, stream);
}

// ---- fanout_scatter_backward (mp_ops.cpp:3103-3166) ------------------------

size_t relm_mp_fanout_scatter_backward_workspace_bytes(int64_t num_edges, int64_t x_rows, int64_t emb,
                                                       relm_mp_dtype dtype)
{
   return op_workspace(num_edges, x_rows, emb, dtype, RELM_MP_MODE_SUM, true);
}

int relm_mp_fanout_scatter_backward(relm_mp_dtype dtype, const void* grad_out, int64_t grad_out_rows, int64_t emb,
                                    const int64_t* src_global_idx, const int64_t* flat_dst, int64_t num_edges,
                                    int64_t x_rows, void* grad_x, void* workspace, size_t workspace_bytes,
                                    void* stream)
{
   int rc;
   if((rc = check_common(dtype, emb, num_edges))) return rc;
   if(x_rows < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "x_rows must be >= 0.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   if(num_edges == 0 || x_rows == 0) return fill_rows(dtype, grad_x, x_rows * emb, false, st);
   OpMem m;
   const size_t need = relm_mp_fanout_scatter_backward_workspace_bytes(num_edges, x_rows, emb, dtype);
   if((rc = split_workspace(workspace, workspace_bytes, need, num_edges, x_rows, m))) return rc;
   relm_mp_plan plan;
   if((rc = plan_build_bounded(
          src_global_idx, flat_dst, num_edges, x_rows, x_rows, grad_out_rows, "src_global_idx", "flat_dst", false,
          m.plan_mem, m.plan_bytes, m.scratch, m.scratch_bytes, st, &plan
       )))
      return rc;
   return planned_reduce(&plan, dtype, kSum, grad_out, nullptr, nullptr, emb, grad_x, m.scratch, m.scratch_bytes, st);
}

// ---- fanin_reduce (mp_ops.cpp:3327-3348 -> 3168-3222 / 3005-3036) ----------

size_t relm_mp_fanin_reduce_workspace_bytes(int64_t num_edges, int64_t dim_size, int64_t emb, relm_mp_dtype dtype,
                                            int mode)
{
   return op_workspace(num_edges, dim_size, emb, dtype, mode, true);
}

int relm_mp_fanin_reduce(relm_mp_dtype dtype, const void* rel_flat, int64_t rel_rows, int64_t emb,
                         const int64_t* flat_src, const int64_t* dst_idx, int64_t num_edges, int64_t dim_size,
                         int mode, void* out, void* workspace, size_t workspace_bytes, void* stream)
{
   int rc;
   if((rc = check_common(dtype, emb, num_edges))) return rc;
   if(dim_size < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "dim_size must be >= 0.");
   if(mode != RELM_MP_MODE_SUM && mode != RELM_MP_MODE_LOGSUMEXP)
      return fail(RELM_MP_ERR_INVALID_ARGUMENT, "Unsupported fanin_reduce mode. Supported: 0=sum, 1=logsumexp.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   if(num_edges == 0 || dim_size == 0)
      return fill_rows(dtype, out, dim_size * emb, mode == RELM_MP_MODE_LOGSUMEXP, st);
   OpMem m;
   const size_t need = relm_mp_fanin_reduce_workspace_bytes(num_edges, dim_size, emb, dtype, mode);
   if((rc = split_workspace(workspace, workspace_bytes, need, num_edges, dim_size, m))) return rc;
   relm_mp_plan plan;
   if((rc = plan_build_bounded(
          dst_idx, flat_src, num_edges, dim_size, dim_size, rel_rows, "dst_idx", "flat_src", true, m.plan_mem,
          m.plan_bytes, m.scratch, m.scratch_bytes, st, &plan
       )))
      return rc;
   return planned_reduce(
      &plan, dtype, mode == RELM_MP_MODE_SUM ? kSum : kLse, rel_flat, nullptr, nullptr, emb, out, m.scratch,
      m.scratch_bytes, st
   );
}

// ---- fanin_reduce_sum_backward (mp_ops.cpp:3224-3284) ----------------------

size_t relm_mp_fanin_reduce_sum_backward_workspace_bytes(int64_t num_edges, int64_t rel_rows, int64_t emb,
                                                         relm_mp_dtype dtype)
{
   return op_workspace(num_edges, rel_rows, emb, dtype, RELM_MP_MODE_SUM, true);
}

int relm_mp_fanin_reduce_sum_backward(relm_mp_dtype dtype, const void* grad_out, int64_t grad_out_rows, int64_t emb,
                                      const int64_t* flat_src, const int64_t* dst_idx, int64_t num_edges,
                                      int64_t rel_rows, void* grad_rel, void* workspace, size_t workspace_bytes,
                                      void* stream)
{
   int rc;
   if((rc = check_common(dtype, emb, num_edges))) return rc;
   if(rel_rows < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "rel_rows must be >= 0.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   if(num_edges == 0 || rel_rows == 0) return fill_rows(dtype, grad_rel, rel_rows * emb, false, st);
   OpMem m;
   const size_t need = relm_mp_fanin_reduce_sum_backward_workspace_bytes(num_edges, rel_rows, emb, dtype);
   if((rc = split_workspace(workspace, workspace_bytes, need, num_edges, rel_rows, m))) return rc;
   relm_mp_plan plan;
   if((rc = plan_build_bounded(
          flat_src, dst_idx, num_edges, rel_rows, rel_rows, grad_out_rows, "flat_src", "dst_idx", false,
          m.plan_mem, m.plan_bytes, m.scratch, m.scratch_bytes, st, &plan
       )))
      return rc;
   return planned_reduce(&plan, dtype, kSum, grad_out, nullptr, nullptr, emb, grad_rel, m.scratch, m.scratch_bytes, st);
}

// ---- fanin_reduce_logsumexp_backward (mp_ops.cpp:3286-3325, 2981-3003) -----

size_t relm_mp_fanin_reduce_logsumexp_backward_workspace_bytes(int64_t num_edges, int64_t rel_rows, int64_t emb,
                                                               relm_mp_dtype dtype)
{
   return op_workspace(num_edges, rel_rows, emb, dtype, RELM_MP_MODE_SUM, true);
}

int relm_mp_fanin_reduce_logsumexp_backward(relm_mp_dtype dtype, const void* grad_out, const void* rel_flat,
                                            int64_t rel_table_rows, const void* out, int64_t dim_size, int64_t emb,
                                            const int64_t* flat_src, const int64_t* dst_idx, int64_t num_edges,
                                            int64_t rel_rows, void* grad_rel, void* workspace,
                                            size_t workspace_bytes, void* stream)
{
   int rc;
   if((rc = check_common(dtype, emb, num_edges))) return rc;
   if(rel_rows < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "rel_rows must be >= 0.");
   if(rel_table_rows < 0 || dim_size < 0) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "sizes must be >= 0.");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   if(num_edges == 0 || rel_rows == 0) return fill_rows(dtype, grad_rel, rel_rows * emb, false, st);
   OpMem m;
   const size_t need = relm_mp_fanin_reduce_logsumexp_backward_workspace_bytes(num_edges, rel_rows, emb, dtype);
   if((rc = split_workspace(workspace, workspace_bytes, need, num_edges, rel_rows, m))) return rc;
   relm_mp_plan plan;
   // flat_src indexes both rel_flat and grad_rel, so it is bounded by the smaller of the two.
   const int64_t bound = rel_table_rows < rel_rows ? rel_table_rows : rel_rows;
   if((rc = plan_build_bounded(
          flat_src, dst_idx, num_edges, rel_rows, bound, dim_size, "flat_src", "dst_idx", false, m.plan_mem,
          m.plan_bytes, m.scratch, m.scratch_bytes, st, &plan
       )))
      return rc;
   return planned_reduce(&plan, dtype, kLseBwd, grad_out, out, rel_flat, emb, grad_rel, m.scratch, m.scratch_bytes, st);
}

}  // extern "C"
