// Plan build: validate an (output index, gather index) pair and lay it out as
// a CSR over the output rows, plus merge-path tile boundaries.
//
// The reference kernels (mp_cuda_kernels.cu:412-649) run one thread per
// (edge, column) and resolve collisions with float atomics. Here every op is a
// segment reduction over output rows instead, so the indices are laid out
// once:
//   1. k_validate   - bounds of both indices (first offending edge, as the
//                     reference CPU loop reports it), sortedness of the output
//                     index and whether it is the identity, int32 copies of
//                     both. An identity output index (edge e writes row e, the
//                     message-row index of a fan-in) skips steps 2 and 3:
//                     k_identity_rows writes row_ptr directly. On request it
//                     also marks the gathered rows (a byte per row, plain
//                     stores), which k_pack_marks turns into the coverage
//                     bitmap and the count of distinct gathered rows: the
//                     gather index repeats a row exactly when that count is
//                     below the edge count. The count travels with the
//                     build's one stats copy, so coverage costs no host sync.
//   2. radix sort   - stable sort of (output row, gathered row) pairs by output
//                     row, only over the bits num_rows needs (skipped when the
//                     output index is already non-decreasing).
//   3. k_mark_ends + inclusive max-scan - row_ptr without atomics: the end of
//                     each non-empty segment is written at row+1, the max-scan
//                     carries it over empty rows.
//   4. k_partition  - merge-path split of the (num_rows + num_edges) items into
//                     equal tiles, so one hub row spreads over many warps and
//                     runs of empty rows cost what their output bytes cost.
#include <climits>
#include <cstdio>
#include <string>

#include "relm_mp_internal.cuh"

namespace relm_mp {

namespace {

struct PlanStats {
   unsigned long long out_bad;     // first edge with an out-of-range output index
   unsigned long long gather_bad;  // first edge with an out-of-range gather index
   unsigned long long covered;     // distinct gathered rows (when marks were requested)
   unsigned int descents;          // warps that saw out_index[e] > out_index[e+1]
   unsigned int not_identity;      // some out_index[e] != e
   unsigned int gather_moved;      // some gather_index[e] != e
};

__global__ void k_init_stats(PlanStats* st)
{
   st->out_bad = ULLONG_MAX;
   st->gather_bad = ULLONG_MAX;
   st->covered = 0;
   st->descents = 0;
   st->not_identity = 0;
   st->gather_moved = 0;
}

constexpr int kValidatePairs = 4;  // edge pairs per thread in the paired validation

__global__ void __launch_bounds__(kThreads) k_validate(const int64_t* __restrict__ key,
                                                       const int64_t* __restrict__ gat, int64_t n,
                                                       int64_t key_bound, int64_t gat_bound,
                                                       uint32_t* __restrict__ key32,
                                                       int32_t* __restrict__ gat32,
                                                       PlanStats* __restrict__ st, bool paired,
                                                       uint8_t* __restrict__ marks)
{
   const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
   bool descent = false;
   bool moved = false;
   bool gmoved = false;
   auto check = [&](int64_t e, int64_t k, int64_t g) __attribute__((always_inline)) {
      gmoved |= g != e;
      if(k < 0 || k >= key_bound) atomicMin(&st->out_bad, (unsigned long long)e);
      if(g < 0 || g >= gat_bound)
         atomicMin(&st->gather_bad, (unsigned long long)e);
      else if(marks)
         marks[g] = 1;  // in bounds: marks holds gat_bound bytes
      moved |= k != e;
   };
   if(paired) {
      // Pairs of edges with 16-byte loads (16-byte aligned indices), kValidatePairs
      // pairs per thread a grid apart, all loads issued before the checks. Odd n:
      // thread 0 also takes the final edge alone.
      const int64_t pairs = n / 2;
      const int64_t T = (int64_t)gridDim.x * blockDim.x;
      longlong2 kk[kValidatePairs], gg[kValidatePairs];
#pragma unroll
      for(int q = 0; q < kValidatePairs; ++q) {
         const int64_t i = t + q * T;
         if(i < pairs) {
            kk[q] = __ldg(reinterpret_cast< const longlong2* >(key) + i);
            gg[q] = gat ? __ldg(reinterpret_cast< const longlong2* >(gat) + i) : make_longlong2(2 * i, 2 * i + 1);
         }
      }
#pragma unroll
      for(int q = 0; q < kValidatePairs; ++q) {
         const int64_t i = t + q * T;
         if(i < pairs) {
            const int64_t e = 2 * i;
            check(e, kk[q].x, gg[q].x);
            check(e + 1, kk[q].y, gg[q].y);
            reinterpret_cast< uint2* >(key32)[i] = make_uint2((uint32_t)kk[q].x, (uint32_t)kk[q].y);
            reinterpret_cast< int2* >(gat32)[i] = make_int2((int32_t)gg[q].x, (int32_t)gg[q].y);
            descent |= kk[q].y < kk[q].x || (e + 2 < n && __ldg(key + e + 2) < kk[q].y);
         }
      }
      if(t == 0 && (n & 1)) {
         const int64_t e = n - 1;
         const int64_t k = key[e];
         const int64_t g = gat ? gat[e] : e;
         check(e, k, g);
         key32[e] = (uint32_t)k;
         gat32[e] = (int32_t)g;
      }
   } else if(t < n) {
      const int64_t k = key[t];
      const int64_t g = gat ? gat[t] : t;
      check(t, k, g);
      key32[t] = (uint32_t)k;
      gat32[t] = (int32_t)g;
      if(t + 1 < n) descent = key[t + 1] < k;
   }
   // One flag write per block at most, and none once the flag is set: a single
   // counter hit by every warp of an unsorted index serialises at L2.
   if(__syncthreads_or(descent) && threadIdx.x == 0 && *((volatile unsigned*)&st->descents) == 0u)
      atomicExch(&st->descents, 1u);
   if(__syncthreads_or(moved) && threadIdx.x == 0 && *((volatile unsigned*)&st->not_identity) == 0u)
      atomicExch(&st->not_identity, 1u);
   if(__syncthreads_or(gmoved) && threadIdx.x == 0 && *((volatile unsigned*)&st->gather_moved) == 0u)
      atomicExch(&st->gather_moved, 1u);
}

// gidx[e] = gather[e] as int32 (a gather index validated elsewhere).
__global__ void __launch_bounds__(kThreads) k_gather32(const int64_t* __restrict__ gather, int64_t n,
                                                       int32_t* __restrict__ gidx)
{
   for(int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x)
      gidx[e] = (int32_t)__ldg(gather + e);
}

// Coverage bitmap from the row marks: word w of `cover` gets bit b set when
// marks[32 w + b] != 0; st->covered += the number of set bits. A thread per
// word, 16-byte loads (marks is 256-byte aligned), the tail word byte by byte.
__global__ void __launch_bounds__(kThreads) k_pack_marks(const uint8_t* __restrict__ marks, int64_t rows,
                                                         uint32_t* __restrict__ cover, PlanStats* __restrict__ st)
{
   const int64_t words = (rows + 31) / 32;
   unsigned long long count = 0;
   for(int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < words; w += (int64_t)gridDim.x * blockDim.x) {
      uint32_t bits = 0;
      if((w + 1) * 32 <= rows) {
         const uint4 a = __ldg(reinterpret_cast< const uint4* >(marks) + 2 * w);
         const uint4 b = __ldg(reinterpret_cast< const uint4* >(marks) + 2 * w + 1);
         const uint32_t q[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
         for(int i = 0; i < 8; ++i)
#pragma unroll
            for(int k = 0; k < 4; ++k) bits |= ((q[i] >> (8 * k)) & 0xffu) ? (1u << (4 * i + k)) : 0u;
      } else {
         for(int64_t r = w * 32; r < rows; ++r) bits |= marks[r] ? (1u << (r - w * 32)) : 0u;
      }
      cover[w] = bits;
      count += (unsigned long long)__popc(bits);
   }
#pragma unroll
   for(int off = 16; off > 0; off >>= 1) count += __shfl_down_sync(0xffffffffu, count, off);
   __shared__ unsigned long long s_count[kThreads / 32];
   if((threadIdx.x & 31) == 0) s_count[threadIdx.x >> 5] = count;
   __syncthreads();
   if(threadIdx.x == 0) {
      unsigned long long total = 0;
      for(int i = 0; i < kThreads / 32; ++i) total += s_count[i];
      if(total) atomicAdd(&st->covered, total);
   }
}

// marks[gidx[j]] = 1 for every edge j of a built plan (validated indices).
__global__ void __launch_bounds__(kThreads) k_mark_gathered(const int32_t* __restrict__ gidx, int64_t n,
                                                            uint8_t* __restrict__ marks)
{
   for(int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x)
      marks[__ldg(gidx + j)] = 1;
}

// Identity output index (out_index[e] == e): row r holds edge r alone for
// r < num_edges, nothing after; flags[2] (rows with edges) = num_edges.
__global__ void __launch_bounds__(kThreads) k_identity_rows(int32_t* __restrict__ row_ptr, int64_t num_rows,
                                                            int64_t num_edges, int32_t* __restrict__ flags)
{
   for(int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r <= num_rows;
       r += (int64_t)gridDim.x * blockDim.x)
      row_ptr[r] = (int32_t)(r < num_edges ? r : num_edges);
   if(blockIdx.x == 0 && threadIdx.x == 0) flags[2] = (int32_t)num_edges;
}

// flags[1] = 1 when some row holds more than kShortRowEdges edges.
__global__ void __launch_bounds__(kThreads) k_long_rows(const int32_t* __restrict__ row_ptr, int64_t num_rows,
                                                        int32_t* __restrict__ flags)
{
   bool long_row = false;
   for(int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < num_rows;
       r += (int64_t)gridDim.x * blockDim.x)
      long_row |= __ldg(row_ptr + r + 1) - __ldg(row_ptr + r) > kShortRowEdges;
   if(__syncthreads_or(long_row) && threadIdx.x == 0 && *((volatile int32_t*)&flags[1]) == 0) flags[1] = 1;
}

// mark[k + 1] = e + 1 where edge e ends the segment of row k (sorted keys);
// flags[0] (has_dups) becomes nonzero if some row holds more than one edge;
// flags[2] counts the rows that hold edges.
__global__ void __launch_bounds__(kThreads) k_mark_ends(const uint32_t* __restrict__ keys,
                                                        int64_t n, int32_t* __restrict__ mark,
                                                        int32_t* __restrict__ flags)
{
   bool dup = false;
   int ends = 0;
   auto visit = [&](int64_t e, uint32_t k, bool last) __attribute__((always_inline)) {
      if(last) {
         mark[(int64_t)k + 1] = (int32_t)(e + 1);
         ++ends;
      } else {
         dup = true;
      }
   };
   const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
   const int64_t stride = (int64_t)gridDim.x * blockDim.x;
   int64_t scalar_from = 0;
   if((reinterpret_cast< uintptr_t >(keys) & 15u) == 0) {
      // Four keys per 16-byte load (the loop is latency-bound with one 4-byte
      // load per thread in flight); the next group's first key comes from L1/L2.
      const int64_t groups = n / 4;
      for(int64_t g = t0; g < groups; g += stride) {
         const uint4 q = __ldg(reinterpret_cast< const uint4* >(keys) + g);
         const int64_t e = g * 4;
         const bool tail = e + 4 >= n;
         const uint32_t nx = tail ? 0u : __ldg(keys + e + 4);
         visit(e, q.x, q.y != q.x);
         visit(e + 1, q.y, q.z != q.y);
         visit(e + 2, q.z, q.w != q.z);
         visit(e + 3, q.w, tail || nx != q.w);
      }
      scalar_from = groups * 4;
   }
   for(int64_t e = scalar_from + t0; e < n; e += stride) {
      const uint32_t k = keys[e];
      visit(e, k, e == n - 1 || keys[e + 1] != k);
   }
   __shared__ int s_ends[kThreads / 32];
#pragma unroll
   for(int off = 16; off > 0; off >>= 1) ends += __shfl_down_sync(0xffffffffu, ends, off);
   if((threadIdx.x & 31) == 0) s_ends[threadIdx.x >> 5] = ends;
   const bool any_dup = __syncthreads_or(dup);
   if(threadIdx.x == 0) {
      int total = 0;
      for(int w = 0; w < kThreads / 32; ++w) total += s_ends[w];
      if(total) atomicAdd(&flags[2], total);
      if(any_dup && *((volatile int32_t*)flags) == 0) flags[0] = 1;
   }
}

// Merge-path search: the split of diagonal d between the row-end list
// (row_ptr[1..num_rows]) and the edge list (0..num_edges-1). Row ends are
// consumed before an edge with the same position, so a split (i, j) means rows
// [0, i) have ended and edges [0, j) are consumed.
__global__ void __launch_bounds__(kThreads) k_partition(const int32_t* __restrict__ row_ptr,
                                                        int64_t num_rows, int64_t num_edges,
                                                        int64_t num_tiles, int tile_items,
                                                        int32_t* __restrict__ tile_row,
                                                        int32_t* __restrict__ tile_edge)
{
   const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
   if(t > num_tiles) return;
   const int64_t total = num_rows + num_edges;
   int64_t d = t * (int64_t)tile_items;
   if(d > total) d = total;
   int64_t lo = d - num_edges > 0 ? d - num_edges : 0;
   int64_t hi = d < num_rows ? d : num_rows;
   while(lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if((int64_t)row_ptr[mid + 1] <= d - mid - 1)
         lo = mid + 1;
      else
         hi = mid;
   }
   tile_row[t] = (int32_t)lo;
   tile_edge[t] = (int32_t)(d - lo);
}


int end_bit_for(int64_t num_rows)
{
   int bits = 1;
   while(bits < 32 && ((int64_t)1 << bits) < num_rows) ++bits;
   return bits;
}


struct PlanLayout {
   int32_t* flags;
   int32_t* gidx;
   int32_t* row_ptr;
   int32_t* tile_row;
   int32_t* tile_edge;
   size_t bytes;
};

PlanLayout plan_layout(void* mem, int64_t num_edges, int64_t num_rows)
{
   Carver c(mem);
   PlanLayout l;
   const int64_t tiles = plan_num_tiles(num_edges, num_rows);
   // [0] has_dups of the output index, [1] gather-cover scratch flag, [2] rows with edges
   l.flags = c.take< int32_t >(4);
   l.gidx = c.take< int32_t >((size_t)num_edges);
   l.row_ptr = c.take< int32_t >((size_t)num_rows + 1);
   l.tile_row = c.take< int32_t >((size_t)tiles + 1);
   l.tile_edge = c.take< int32_t >((size_t)tiles + 1);
   l.bytes = c.used;
   return l;
}

struct ScratchLayout {
   PlanStats* stats;
   uint8_t* marks;  // gathered-row marks (cover_rows bytes), when coverage is requested
   uint32_t* key_in;
   uint32_t* key_alt;
   int32_t* val_alt;
   int32_t* mark;
   void* sort_temp;
   size_t sort_bytes;
   void* scan_temp;
   size_t scan_bytes;
   size_t bytes;
};

ScratchLayout scratch_layout(void* mem, int64_t num_edges, int64_t num_rows, int64_t cover_rows = 0)
{
   Carver c(mem);
   ScratchLayout l;
   l.stats = c.take< PlanStats >(1);
   l.marks = cover_rows > 0 ? c.take< uint8_t >((size_t)cover_rows) : nullptr;
   l.key_in = c.take< uint32_t >((size_t)num_edges);
   l.key_alt = c.take< uint32_t >((size_t)num_edges);
   l.val_alt = c.take< int32_t >((size_t)num_edges);
   l.mark = c.take< int32_t >((size_t)num_rows + 1);
   l.sort_bytes = radix_sort_temp_bytes(num_edges, end_bit_for(num_rows));
   l.sort_temp = c.take< char >(l.sort_bytes);
   l.scan_bytes = scan_i32_temp_bytes(num_rows + 1);
   l.scan_temp = c.take< char >(l.scan_bytes);
   l.bytes = c.used;
   return l;
}

unsigned grid_for(int64_t n, int threads = kThreads)
{
   return (unsigned)((n + threads - 1) / threads);
}

}  // namespace

int plan_tile_items(int64_t num_edges, int64_t num_rows)
{
   const int64_t total = num_edges + num_rows;
   int64_t items = (total + kTargetTiles - 1) / kTargetTiles;
   items = (items + 31) / 32 * 32;
   if(items < kMinTileItems) items = kMinTileItems;
   if(items > kMaxTileItems) items = kMaxTileItems;
   return (int)items;
}

int64_t plan_num_tiles(int64_t num_edges, int64_t num_rows)
{
   const int items = plan_tile_items(num_edges, num_rows);
   return (num_edges + num_rows + items - 1) / items;
}

int plan_build_bounded(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                       int64_t num_rows, int64_t out_bound, int64_t gather_rows,
                       const char* out_name, const char* gather_name, bool gather_checked_first,
                       void* plan_mem, size_t plan_bytes, void* scratch, size_t scratch_bytes,
                       cudaStream_t stream, relm_mp_plan* plan, uint32_t* cover, int* gather_repeats,
                       int64_t* gather_covered, BuildPhase phase, void* host_stats)
{
   if(!plan) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan must not be NULL.");
   if((phase == kBuildStart || phase == kBuildFinish) && !host_stats)
      return fail(RELM_MP_ERR_INVALID_ARGUMENT, "host_stats must not be NULL.");
   if(num_edges < 0 || num_rows < 0 || gather_rows < 0)
      return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan sizes must be >= 0.");
   if(num_edges + num_rows >= (int64_t)INT32_MAX || gather_rows >= (int64_t)INT32_MAX)
      return fail(
         RELM_MP_ERR_UNSUPPORTED, "relm_mp supports num_edges + num_rows < 2^31 and < 2^31 gathered rows."
      );
   if(num_edges > 0 && !out_index) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "out_index must not be NULL.");
   if(cover && !gather_repeats) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "gather_repeats must not be NULL.");
   const PlanLayout pl = plan_layout(plan_mem, num_edges, num_rows);
   const ScratchLayout sl = scratch_layout(scratch, num_edges, num_rows, cover ? gather_rows : 0);
   if(!plan_mem || plan_bytes < pl.bytes)
      return fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, "plan memory is smaller than relm_mp_plan_bytes().");
   if(!scratch || scratch_bytes < sl.bytes)
      return fail(
         RELM_MP_ERR_WORKSPACE_TOO_SMALL,
         cover ? "plan scratch is smaller than relm_mp_plan_cover_scratch_bytes()."
               : "plan scratch is smaller than relm_mp_plan_scratch_bytes()."
      );
   const char* oname = out_name ? out_name : "out_index";
   const char* gname = gather_name ? gather_name : "gather_index";

   const int64_t tiles = plan_num_tiles(num_edges, num_rows);
   *plan = relm_mp_plan{};
   plan->num_edges = num_edges;
   plan->num_rows = num_rows;
   plan->gather_rows = gather_rows;
   plan->num_tiles = tiles;
   plan->tile_items = plan_tile_items(num_edges, num_rows);
   plan->row_ptr = pl.row_ptr;
   plan->gidx = pl.gidx;
   plan->tile_row = pl.tile_row;
   plan->tile_edge = pl.tile_edge;
   plan->device_flags = pl.flags;

   int rc;
   // The sort's values ping-pong between val_alt and gidx, one pass per up to
   // 11 key bits; with an odd pass count the sorted values land in the plan's
   // gidx when validation writes them to val_alt first.
   const int sort_passes = radix_sort_passes(end_bit_for(num_rows));
   int32_t* gather32 = (sort_passes & 1) ? sl.val_alt : pl.gidx;
   // The validation's statistics reach the host through `host`: the build's
   // own (synchronous) copy, or the caller's pinned buffer when the build is
   // split (start: validate and queue the copy; finish: after the caller's
   // wait, check them and lay the plan out).
   PlanStats local{};
   PlanStats& host = (phase == kBuildAll || phase == kBuildTrusted) ? local : *static_cast< PlanStats* >(host_stats);
   if(phase == kBuildTrusted) {
      // validated elsewhere against these bounds: the validation kernel only
      // narrows both indices (no bound can fail), its flags stay on the device
      if(num_edges > 0) {
         const bool paired = (reinterpret_cast< uintptr_t >(out_index) & 15u) == 0 &&
                             (reinterpret_cast< uintptr_t >(gather_index) & 15u) == 0 &&
                             (reinterpret_cast< uintptr_t >(sl.key_in) & 7u) == 0 &&
                             (reinterpret_cast< uintptr_t >(gather32) & 7u) == 0;
         k_init_stats<<< 1, 1, 0, stream >>>(sl.stats);
         if((rc = check_launch("k_init_stats"))) return rc;
         k_validate<<< grid_for(paired ? (num_edges / 2 + kValidatePairs - 1) / kValidatePairs + 1 : num_edges),
                    kThreads, 0, stream >>>(
            out_index, gather_index, num_edges, INT64_MAX, INT64_MAX, sl.key_in, gather32, sl.stats, paired, nullptr
         );
         if((rc = check_launch("k_validate"))) return rc;
      }
      local.out_bad = ULLONG_MAX;
      local.gather_bad = ULLONG_MAX;
      local.descents = 1;
      local.not_identity = 1;
      local.gather_moved = 1;
   } else if(phase != kBuildFinish) {
      k_init_stats<<< 1, 1, 0, stream >>>(sl.stats);
      if((rc = check_launch("k_init_stats"))) return rc;
      if(cover &&
         (rc = check_cuda(cudaMemsetAsync(sl.marks, 0, (size_t)gather_rows, stream), "marks memset")))
         return rc;
      if(num_edges > 0) {
         const bool paired = (reinterpret_cast< uintptr_t >(out_index) & 15u) == 0 &&
                             (reinterpret_cast< uintptr_t >(gather_index) & 15u) == 0 &&
                             (reinterpret_cast< uintptr_t >(sl.key_in) & 7u) == 0 &&
                             (reinterpret_cast< uintptr_t >(gather32) & 7u) == 0;
         k_validate<<< grid_for(paired ? (num_edges / 2 + kValidatePairs - 1) / kValidatePairs + 1 : num_edges),
                    kThreads, 0, stream >>>(
            out_index, gather_index, num_edges, out_bound, gather_rows, sl.key_in, gather32, sl.stats, paired,
            cover ? sl.marks : nullptr
         );
         if((rc = check_launch("k_validate"))) return rc;
      }
      if(cover) {
         const int64_t words = (int64_t)relm_mp_cover_words(gather_rows);
         if(gather_rows > 0) {
            unsigned grid = grid_for(words);
            if(grid > 148u * 8u) grid = 148u * 8u;
            k_pack_marks<<< grid, kThreads, 0, stream >>>(sl.marks, gather_rows, cover, sl.stats);
            if((rc = check_launch("k_pack_marks"))) return rc;
         } else if((rc = check_cuda(cudaMemsetAsync(cover, 0, sizeof(uint32_t), stream), "cover memset"))) {
            return rc;
         }
      }
      if((rc = check_cuda(
             cudaMemcpyAsync(&host, sl.stats, sizeof(PlanStats), cudaMemcpyDeviceToHost, stream),
             "plan stats copy"
          )))
         return rc;
      if(phase == kBuildStart) return RELM_MP_OK;
      if((rc = check_cuda(cudaStreamSynchronize(stream), "plan stats sync"))) return rc;
   }  // validation

   if(host.out_bad != ULLONG_MAX || host.gather_bad != ULLONG_MAX) {
      bool use_gather;
      if(host.out_bad == host.gather_bad)
         use_gather = gather_checked_first;
      else
         use_gather = host.gather_bad < host.out_bad;
      const unsigned long long pos = use_gather ? host.gather_bad : host.out_bad;
      const int64_t* arr = use_gather ? gather_index : out_index;
      int64_t value = (int64_t)pos;  // a NULL (identity) gather index gathers row e at edge e
      if(arr) {
         if((rc = check_cuda(
                cudaMemcpyAsync(&value, arr + pos, sizeof(int64_t), cudaMemcpyDeviceToHost, stream),
                "bad index copy"
             )))
            return rc;
         if((rc = check_cuda(cudaStreamSynchronize(stream), "bad index sync"))) return rc;
      }
      char msg[256];
      snprintf(
         msg,
         sizeof msg,
         "%s index out of bounds: %lld not in [0, %lld).",
         use_gather ? gname : oname,
         (long long)value,
         (long long)(use_gather ? gather_rows : out_bound)
      );
      return fail(RELM_MP_ERR_INDEX_OUT_OF_RANGE, msg);
   }
   if(cover) *gather_repeats = host.covered != (unsigned long long)num_edges;
   if(cover && gather_covered) *gather_covered = (int64_t)host.covered;
   if(num_edges > 0 && host.gather_moved == 0) plan->flags |= RELM_MP_PLAN_GATHER_IDENTITY;
   auto gidx_home = [&]() -> int {  // the unsorted gather values, into the plan's gidx
      if(gather32 == pl.gidx || num_edges == 0) return RELM_MP_OK;
      return check_cuda(cudaMemcpyAsync(pl.gidx, gather32, (size_t)num_edges * sizeof(int32_t),
                                        cudaMemcpyDeviceToDevice, stream),
                        "gidx copy");
   };

   if(host.not_identity == 0) {  // edge e is row e: no sort, no segment scan
      if((rc = gidx_home())) return rc;
      plan->flags |= RELM_MP_PLAN_SORTED_INPUT;
      if((rc = check_cuda(cudaMemsetAsync(pl.flags, 0, 4 * sizeof(int32_t), stream), "flags memset"))) return rc;
      unsigned grid = grid_for(num_rows + 1);
      if(grid > 148u * 8u) grid = 148u * 8u;
      k_identity_rows<<< grid, kThreads, 0, stream >>>(pl.row_ptr, num_rows, num_edges, pl.flags);
      if((rc = check_launch("k_identity_rows"))) return rc;
      k_partition<<< grid_for(tiles + 1), kThreads, 0, stream >>>(
         pl.row_ptr, num_rows, num_edges, tiles, plan->tile_items, pl.tile_row, pl.tile_edge
      );
      return check_launch("k_partition");
   }

   const uint32_t* sorted_keys = sl.key_in;
   if(host.descents == 0) {
      plan->flags |= RELM_MP_PLAN_SORTED_INPUT;
      if((rc = gidx_home())) return rc;
   } else {
      int32_t* val_other = gather32 == pl.gidx ? sl.val_alt : pl.gidx;
      bool in_alt = false;
      if((rc = radix_sort_pairs(sl.key_in, sl.key_alt, gather32, val_other, num_edges, end_bit_for(num_rows),
                                sl.sort_temp, sl.sort_bytes, stream, &in_alt)))
         return rc;
      sorted_keys = in_alt ? sl.key_alt : sl.key_in;
      const int32_t* sorted_vals = in_alt ? val_other : gather32;
      if(sorted_vals != pl.gidx) {
         if((rc = check_cuda(
                cudaMemcpyAsync(
                   pl.gidx, sorted_vals, (size_t)num_edges * sizeof(int32_t), cudaMemcpyDeviceToDevice, stream
                ),
                "gidx copy"
             )))
            return rc;
      }
   }

   if((rc = check_cuda(
          cudaMemsetAsync(sl.mark, 0, ((size_t)num_rows + 1) * sizeof(int32_t), stream), "mark memset"
       )))
      return rc;
   if((rc = check_cuda(cudaMemsetAsync(pl.flags, 0, 4 * sizeof(int32_t), stream), "flags memset"))) return rc;
   if(num_edges > 0) {
      unsigned grid = grid_for(num_edges);
      if(grid > 148u * 8u) grid = 148u * 8u;
      k_mark_ends<<< grid, kThreads, 0, stream >>>(sorted_keys, num_edges, sl.mark, pl.flags);
      if((rc = check_launch("k_mark_ends"))) return rc;
   }
   if((rc = scan_max_inclusive(sl.mark, pl.row_ptr, num_rows + 1, sl.scan_temp, sl.scan_bytes, stream))) return rc;
   k_partition<<< grid_for(tiles + 1), kThreads, 0, stream >>>(
      pl.row_ptr, num_rows, num_edges, tiles, plan->tile_items, pl.tile_row, pl.tile_edge
   );
   if((rc = check_launch("k_partition"))) return rc;
   if(num_edges > 0) {
      unsigned grid = grid_for(num_rows);
      if(grid > 148u * 4u) grid = 148u * 4u;
      k_long_rows<<< grid, kThreads, 0, stream >>>(pl.row_ptr, num_rows, pl.flags);
      if((rc = check_launch("k_long_rows"))) return rc;
   }
   return RELM_MP_OK;
}

}  // namespace relm_mp

extern "C" {

size_t relm_mp_plan_bytes(int64_t num_edges, int64_t num_rows)
{
   if(num_edges < 0 || num_rows < 0) return 0;
   return relm_mp::plan_layout(nullptr, num_edges, num_rows).bytes;
}

size_t relm_mp_plan_scratch_bytes(int64_t num_edges, int64_t num_rows)
{
   if(num_edges < 0 || num_rows < 0) return 0;
   return relm_mp::scratch_layout(nullptr, num_edges, num_rows).bytes;
}

int relm_mp_plan_build(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                       int64_t num_rows, int64_t gather_rows, const char* out_index_name,
                       const char* gather_index_name, void* plan_mem, size_t plan_bytes,
                       void* scratch, size_t scratch_bytes, void* stream, relm_mp_plan* plan)
{
   return relm_mp::plan_build_bounded(
      out_index, gather_index, num_edges, num_rows, num_rows, gather_rows, out_index_name,
      gather_index_name, false, plan_mem, plan_bytes, scratch, scratch_bytes,
      static_cast< cudaStream_t >(stream), plan
   );
}

size_t relm_mp_plan_gather_cover_scratch_bytes(const relm_mp_plan* plan)
{
   if(!plan) return 0;
   relm_mp::Carver c(nullptr);
   c.take< relm_mp::PlanStats >(1);
   c.take< uint8_t >((size_t)plan->gather_rows);
   return c.used;
}

int relm_mp_plan_gather_cover_ex(const relm_mp_plan* plan, uint32_t* cover, int* has_dups, int64_t* covered_rows,
                                 void* scratch, size_t scratch_bytes, void* stream)
{
   using namespace relm_mp;
   if(!plan || !cover || !has_dups) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan, cover and has_dups must not be NULL.");
   if(!scratch || scratch_bytes < relm_mp_plan_gather_cover_scratch_bytes(plan))
      return fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, "scratch is smaller than relm_mp_plan_gather_cover_scratch_bytes().");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   Carver c(scratch);
   PlanStats* stats = c.take< PlanStats >(1);
   uint8_t* marks = c.take< uint8_t >((size_t)plan->gather_rows);
   int rc;
   k_init_stats<<< 1, 1, 0, st >>>(stats);
   if((rc = check_launch("k_init_stats"))) return rc;
   if(plan->gather_rows == 0) {
      *has_dups = 0;
      if(covered_rows) *covered_rows = 0;
      return check_cuda(cudaMemsetAsync(cover, 0, sizeof(uint32_t), st), "cover memset");
   }
   if((rc = check_cuda(cudaMemsetAsync(marks, 0, (size_t)plan->gather_rows, st), "marks memset"))) return rc;
   if(plan->num_edges > 0) {
      unsigned grid = grid_for(plan->num_edges);
      if(grid > 148u * 16u) grid = 148u * 16u;
      k_mark_gathered<<< grid, kThreads, 0, st >>>(plan->gidx, plan->num_edges, marks);
      if((rc = check_launch("k_mark_gathered"))) return rc;
   }
   unsigned grid = grid_for((int64_t)relm_mp_cover_words(plan->gather_rows));
   if(grid > 148u * 8u) grid = 148u * 8u;
   k_pack_marks<<< grid, kThreads, 0, st >>>(marks, plan->gather_rows, cover, stats);
   if((rc = check_launch("k_pack_marks"))) return rc;
   unsigned long long covered = 0;
   if((rc = check_cuda(cudaMemcpyAsync(&covered, &stats->covered, sizeof covered, cudaMemcpyDeviceToHost, st),
                       "cover count copy")))
      return rc;
   if((rc = check_cuda(cudaStreamSynchronize(st), "cover sync"))) return rc;
   *has_dups = covered != (unsigned long long)plan->num_edges;
   if(covered_rows) *covered_rows = (int64_t)covered;
   return RELM_MP_OK;
}

size_t relm_mp_plan_cover_scratch_bytes(int64_t num_edges, int64_t num_rows, int64_t gather_rows)
{
   if(num_edges < 0 || num_rows < 0 || gather_rows < 0) return 0;
   return relm_mp::scratch_layout(nullptr, num_edges, num_rows, gather_rows).bytes;
}

int relm_mp_plan_build_cover(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                             int64_t num_rows, int64_t out_bound, int64_t gather_rows, const char* out_index_name,
                             const char* gather_index_name, int gather_checked_first, void* plan_mem,
                             size_t plan_bytes, void* scratch, size_t scratch_bytes, uint32_t* cover,
                             int* gather_repeats, int64_t* gather_covered, void* stream, relm_mp_plan* plan)
{
   if(out_bound < 0 || out_bound > num_rows)
      return relm_mp::fail(RELM_MP_ERR_INVALID_ARGUMENT, "out_bound must be in [0, num_rows].");
   if(!cover || !gather_repeats)
      return relm_mp::fail(RELM_MP_ERR_INVALID_ARGUMENT, "cover and gather_repeats must not be NULL.");
   return relm_mp::plan_build_bounded(
      out_index, gather_index, num_edges, num_rows, out_bound, gather_rows, out_index_name, gather_index_name,
      gather_checked_first != 0, plan_mem, plan_bytes, scratch, scratch_bytes, static_cast< cudaStream_t >(stream),
      plan, cover, gather_repeats, gather_covered
   );
}

size_t relm_mp_plan_stats_bytes(void) { return sizeof(relm_mp::PlanStats); }

int relm_mp_plan_build_identity(const int64_t* gather_index, int64_t num_edges, int64_t num_rows,
                                int64_t gather_rows, void* plan_mem, size_t plan_bytes, void* stream,
                                relm_mp_plan* plan)
{
   using namespace relm_mp;
   if(!plan) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "plan must not be NULL.");
   if(num_edges < 0 || num_rows < num_edges || gather_rows < 0)
      return fail(RELM_MP_ERR_INVALID_ARGUMENT, "relm_mp_plan_build_identity needs 0 <= num_edges <= num_rows.");
   if(num_edges + num_rows >= (int64_t)INT32_MAX || gather_rows >= (int64_t)INT32_MAX)
      return fail(
         RELM_MP_ERR_UNSUPPORTED, "relm_mp supports num_edges + num_rows < 2^31 and < 2^31 gathered rows."
      );
   if(num_edges > 0 && !gather_index) return fail(RELM_MP_ERR_INVALID_ARGUMENT, "gather_index must not be NULL.");
   const PlanLayout pl = plan_layout(plan_mem, num_edges, num_rows);
   if(!plan_mem || plan_bytes < pl.bytes)
      return fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, "plan memory is smaller than relm_mp_plan_bytes().");
   cudaStream_t st = static_cast< cudaStream_t >(stream);
   const int64_t tiles = plan_num_tiles(num_edges, num_rows);
   *plan = relm_mp_plan{};
   plan->num_edges = num_edges;
   plan->num_rows = num_rows;
   plan->gather_rows = gather_rows;
   plan->num_tiles = tiles;
   plan->tile_items = plan_tile_items(num_edges, num_rows);
   plan->row_ptr = pl.row_ptr;
   plan->gidx = pl.gidx;
   plan->tile_row = pl.tile_row;
   plan->tile_edge = pl.tile_edge;
   plan->device_flags = pl.flags;
   // every row holds at most one edge: the row facts are known without a device pass
   plan->flags = RELM_MP_PLAN_SORTED_INPUT | RELM_MP_PLAN_FLAGS_KNOWN;
   int rc;
   if((rc = check_cuda(cudaMemsetAsync(pl.flags, 0, 4 * sizeof(int32_t), st), "flags memset"))) return rc;
   if(num_edges > 0) {
      unsigned grid = grid_for(num_edges);
      if(grid > 148u * 16u) grid = 148u * 16u;
      k_gather32<<< grid, kThreads, 0, st >>>(gather_index, num_edges, pl.gidx);
      if((rc = check_launch("k_gather32"))) return rc;
   }
   unsigned grid = grid_for(num_rows + 1);
   if(grid > 148u * 8u) grid = 148u * 8u;
   k_identity_rows<<< grid, kThreads, 0, st >>>(pl.row_ptr, num_rows, num_edges, pl.flags);
   if((rc = check_launch("k_identity_rows"))) return rc;
   k_partition<<< grid_for(tiles + 1), kThreads, 0, st >>>(
      pl.row_ptr, num_rows, num_edges, tiles, plan->tile_items, pl.tile_row, pl.tile_edge
   );
   return check_launch("k_partition");
}

int relm_mp_plan_build_start(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                             int64_t num_rows, int64_t out_bound, int64_t gather_rows, void* plan_mem,
                             size_t plan_bytes, void* scratch, size_t scratch_bytes, void* host_stats, void* stream)
{
   if(out_bound < 0 || out_bound > num_rows)
      return relm_mp::fail(RELM_MP_ERR_INVALID_ARGUMENT, "out_bound must be in [0, num_rows].");
   relm_mp_plan plan;
   return relm_mp::plan_build_bounded(
      out_index, gather_index, num_edges, num_rows, out_bound, gather_rows, nullptr, nullptr, false, plan_mem,
      plan_bytes, scratch, scratch_bytes, static_cast< cudaStream_t >(stream), &plan, nullptr, nullptr, nullptr,
      relm_mp::kBuildStart, host_stats
   );
}

int relm_mp_plan_build_trusted(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                               int64_t num_rows, int64_t gather_rows, void* plan_mem, size_t plan_bytes,
                               void* scratch, size_t scratch_bytes, void* stream, relm_mp_plan* plan)
{
   if(num_edges > 0 && !gather_index)
      return relm_mp::fail(RELM_MP_ERR_INVALID_ARGUMENT, "gather_index must not be NULL.");
   return relm_mp::plan_build_bounded(
      out_index, gather_index, num_edges, num_rows, num_rows, gather_rows, nullptr, nullptr, false, plan_mem,
      plan_bytes, scratch, scratch_bytes, static_cast< cudaStream_t >(stream), plan, nullptr, nullptr, nullptr,
      relm_mp::kBuildTrusted, nullptr
   );
}

int relm_mp_plan_build_finish(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                              int64_t num_rows, int64_t out_bound, int64_t gather_rows, const char* out_index_name,
                              const char* gather_index_name, int gather_checked_first, void* plan_mem,
                              size_t plan_bytes, void* scratch, size_t scratch_bytes, const void* host_stats,
                              void* stream, relm_mp_plan* plan)
{
   if(out_bound < 0 || out_bound > num_rows)
      return relm_mp::fail(RELM_MP_ERR_INVALID_ARGUMENT, "out_bound must be in [0, num_rows].");
   return relm_mp::plan_build_bounded(
      out_index, gather_index, num_edges, num_rows, out_bound, gather_rows, out_index_name, gather_index_name,
      gather_checked_first != 0, plan_mem, plan_bytes, scratch, scratch_bytes, static_cast< cudaStream_t >(stream),
      plan, nullptr, nullptr, nullptr, relm_mp::kBuildFinish, const_cast< void* >(host_stats)
   );
}

int relm_mp_plan_build_ex(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                          int64_t num_rows, int64_t out_bound, int64_t gather_rows, const char* out_index_name,
                          const char* gather_index_name, int gather_checked_first, void* plan_mem,
                          size_t plan_bytes, void* scratch, size_t scratch_bytes, void* stream, relm_mp_plan* plan)
{
   if(out_bound < 0 || out_bound > num_rows)
      return relm_mp::fail(RELM_MP_ERR_INVALID_ARGUMENT, "out_bound must be in [0, num_rows].");
   return relm_mp::plan_build_bounded(
      out_index, gather_index, num_edges, num_rows, out_bound, gather_rows, out_index_name,
      gather_index_name, gather_checked_first != 0, plan_mem, plan_bytes, scratch, scratch_bytes,
      static_cast< cudaStream_t >(stream), plan
   );
}

}  // extern "C"
