// Plan-build sort and scans, written for the plan's shapes:
//
//   radix_sort_pairs - stable LSD radix sort of (uint32 key, int32 value)
//                      pairs over the key bits a plan needs (the output row,
//                      < num_rows), in as few passes of at most 10 bits as the
//                      width allows: 2 passes for up to 2^20 rows, 3 for up to
//                      2^30 (10-bit digits keep two CTAs per SM and runs of
//                      about 8 items per digit and sub-tile; 11-bit digits
//                      measured slower on 2^22 rows). Each pass is
//                        k_sort_hist    digit counts of every CTA's item range,
//                                       laid out digit-major [digit][cta];
//                        exclusive scan of those counts -> every (digit, CTA)
//                                       pair's first output position;
//                        k_sort_scatter each CTA walks its range in sub-tiles
//                                       of 8192 items: a warp ranks its 512
//                                       items in order (lane masks of equal
//                                       digits OR-ed together in shared
//                                       memory, per-warp counters), the
//                                       sub-tile is reordered by digit in
//                                       shared memory and written out in
//                                       digit runs with coalesced stores.
//                      Items keep their input order within a digit (ranks
//                      follow item order within warps, warps, sub-tiles and
//                      CTAs), so the sort is stable and the plan's edge order
//                      within a row is the input order, run to run.
//   scan_i32         - exclusive sum or inclusive max scan of int32 arrays
//                      (block totals, then each block adds up the totals
//                      before it and scans its own chunk).
//
// No atomics on global memory, no inter-CTA waiting.
#include <climits>

#include "relm_mp_internal.cuh"

namespace relm_mp {

namespace {

// Threads of a sort CTA (512 or 1024; a build-time setting of tuning builds).
#ifndef RELM_MP_SORT_THREADS
#define RELM_MP_SORT_THREADS 512
#endif
constexpr int kSortThreads = RELM_MP_SORT_THREADS;
constexpr int kSortCtasPerSm = kSortThreads <= 512 ? 2 : 1;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortPerThread = 16;
constexpr int kSortSub = kSortThreads * kSortPerThread;  // items per sub-tile
constexpr int kSortMaxBits = 10;  // digit bits per pass
constexpr int kScanThreads = 512;
constexpr int kScanPerThread = 8;
constexpr int kScanChunk = kScanThreads * kScanPerThread;

struct SumOp {
   static constexpr int32_t identity = 0;
   __device__ __forceinline__ int32_t operator()(int32_t a, int32_t b) const { return a + b; }
};
struct MaxOp32 {
   static constexpr int32_t identity = INT_MIN;
   __device__ __forceinline__ int32_t operator()(int32_t a, int32_t b) const { return a > b ? a : b; }
};

// Exclusive scan of one value per thread over the block; *total gets the
// reduction of all of them. `wtot` holds one entry per warp (shared memory).
template < class Op >
__device__ __forceinline__ int32_t block_exclusive(int32_t v, int32_t* wtot, int32_t* total)
{
   const Op op;
   const int lane = threadIdx.x & 31;
   const int w = threadIdx.x >> 5;
   const int nw = blockDim.x >> 5;
   int32_t x = v;
#pragma unroll
   for(int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if(lane >= o) x = op(x, y);
   }
   int32_t excl = __shfl_up_sync(0xffffffffu, x, 1);
   if(lane == 0) excl = Op::identity;
   if(lane == 31) wtot[w] = x;
   __syncthreads();
   if(w == 0) {
      int32_t t = lane < nw ? wtot[lane] : Op::identity;
#pragma unroll
      for(int o = 1; o < 32; o <<= 1) {
         const int32_t y = __shfl_up_sync(0xffffffffu, t, o);
         if(lane >= o) t = op(t, y);
      }
      if(lane < nw) wtot[lane] = t;
   }
   __syncthreads();
   const int32_t before = w > 0 ? wtot[w - 1] : Op::identity;
   *total = wtot[nw - 1];
   __syncthreads();  // wtot may be reused right away
   return op(before, excl);
}

// ---- scan -----------------------------------------------------------------------------

template < class Op >
__global__ void __launch_bounds__(kScanThreads) k_scan_reduce(const int32_t* __restrict__ in, int64_t n,
                                                              int32_t* __restrict__ part)
{
   __shared__ int32_t wtot[kScanThreads / 32];
   const Op op;
   const int64_t base = (int64_t)blockIdx.x * kScanChunk + (int64_t)threadIdx.x * kScanPerThread;
   int32_t acc = Op::identity;
#pragma unroll
   for(int i = 0; i < kScanPerThread; ++i)
      if(base + i < n) acc = op(acc, in[base + i]);
   int32_t total;
   block_exclusive< Op >(acc, wtot, &total);
   if(threadIdx.x == 0) part[blockIdx.x] = total;
}

template < class Op, bool INCLUSIVE >
__global__ void __launch_bounds__(kScanThreads) k_scan_apply(const int32_t* __restrict__ in, int64_t n,
                                                             const int32_t* __restrict__ part,
                                                             int32_t* __restrict__ out)
{
   __shared__ int32_t wtot[kScanThreads / 32];
   const Op op;
   const int64_t base = (int64_t)blockIdx.x * kScanChunk + (int64_t)threadIdx.x * kScanPerThread;
   int32_t v[kScanPerThread];
   int32_t acc = Op::identity;
#pragma unroll
   for(int i = 0; i < kScanPerThread; ++i) {
      v[i] = base + i < n ? in[base + i] : Op::identity;
      acc = op(acc, v[i]);
   }
   // the reduction of the blocks before this one (their totals in `part`)
   int32_t carry = Op::identity;
   for(int64_t b = threadIdx.x; b < (int64_t)blockIdx.x; b += kScanThreads) carry = op(carry, part[b]);
   int32_t before;
   block_exclusive< Op >(carry, wtot, &before);
   int32_t total;
   int32_t run = op(before, block_exclusive< Op >(acc, wtot, &total));
#pragma unroll
   for(int i = 0; i < kScanPerThread; ++i) {
      if(base + i < n) {
         if(INCLUSIVE) {
            run = op(run, v[i]);
            out[base + i] = run;
         } else {
            out[base + i] = run;
            run = op(run, v[i]);
         }
      }
   }
}

int64_t scan_blocks(int64_t n) { return (n + kScanChunk - 1) / kScanChunk; }

// ---- radix sort -----------------------------------------------------------------------

struct SortShape {
   int passes;
   int bits[32];
   int shift[32];
   int subs;      // sub-tiles per CTA
   int64_t ctas;  // CTAs of a pass (the same item ranges in the histogram and the scatter)
};

SortShape sort_shape(int64_t n, int end_bit)
{
   SortShape s{};
   if(end_bit < 1) end_bit = 1;
   s.passes = (end_bit + kSortMaxBits - 1) / kSortMaxBits;
   int done = 0;
   for(int i = 0; i < s.passes; ++i) {
      const int left = end_bit - done;
      const int b = (left + (s.passes - i) - 1) / (s.passes - i);
      s.bits[i] = b;
      s.shift[i] = done;
      done += b;
   }
   // about two CTAs per SM, at most 16 sub-tiles each
   const int64_t sub_tiles = (n + kSortSub - 1) / kSortSub;
   int64_t subs = (sub_tiles + kSortCtasPerSm * 148 - 1) / (kSortCtasPerSm * 148);
   if(subs < 1) subs = 1;
   if(subs > 16) subs = 16;
   s.subs = (int)subs;
   s.ctas = (sub_tiles + subs - 1) / subs;
   if(s.ctas < 1) s.ctas = 1;
   return s;
}

__device__ __forceinline__ unsigned lanemask_lt()
{
   unsigned m;
   asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
   return m;
}

// Bulk prefetch of items [from, from + count) of a 32-bit array into L2 (the
// copy engine fetches it while the CTA works on the sub-tile before), for a
// 16-byte aligned start; the last count % 4 items are left out.
template < class T >
__device__ __forceinline__ void prefetch_items_l2(const T* a, int64_t from, int64_t count)
{
   static_assert(sizeof(T) == 4, "32-bit items");
   const T* p = a + from;
   const uint32_t bytes = (uint32_t)(count * 4) & ~15u;
   if(bytes == 0 || (reinterpret_cast< uintptr_t >(p) & 15u)) return;
   asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Digit counts of CTA c's items [c * subs * kSortSub, ...): ghist[d * ctas + c].
// Each sub-tile's keys are loaded up front (16 independent loads per thread)
// and counted with shared-memory atomics into 4 sub-histograms (warp mod 4),
// which spreads the collisions of a hot digit over more addresses.
template < int DB >
__global__ void __launch_bounds__(kSortThreads) k_sort_hist(const uint32_t* __restrict__ keys, int64_t n, int shift,
                                                            int32_t* __restrict__ ghist, int64_t ctas, int subs)
{
   constexpr int D = 1 << DB;
   __shared__ int32_t h[4][D];
   for(int d = threadIdx.x; d < 4 * D; d += kSortThreads) (&h[0][0])[d] = 0;
   __syncthreads();
   const int lane = threadIdx.x & 31;
   const int w = threadIdx.x >> 5;
   int32_t* hw = h[w & 3];
   const int64_t c = blockIdx.x;
   for(int sub = 0; sub < subs; ++sub) {
      const int64_t base = (c * subs + sub) * (int64_t)kSortSub;
      if(base >= n) break;
      const int subn = (n - base) < kSortSub ? (int)(n - base) : kSortSub;
      if(threadIdx.x == 0 && sub + 1 < subs && base + kSortSub < n)
         prefetch_items_l2(keys, base + kSortSub, n - base - kSortSub < kSortSub ? n - base - kSortSub : kSortSub);
      uint32_t k[kSortPerThread];
#pragma unroll
      for(int r = 0; r < kSortPerThread; ++r) {
         const int idx = w * (kSortSub / kSortWarps) + r * 32 + lane;
         k[r] = idx < subn ? __ldg(keys + base + idx) : 0u;
      }
#pragma unroll
      for(int r = 0; r < kSortPerThread; ++r) {
         const int idx = w * (kSortSub / kSortWarps) + r * 32 + lane;
         if(idx < subn) atomicAdd(&hw[(k[r] >> shift) & (D - 1)], 1);
      }
   }
   __syncthreads();
   for(int d = threadIdx.x; d < D; d += kSortThreads)
      ghist[(int64_t)d * ctas + c] = h[0][d] + h[1][d] + h[2][d] + h[3][d];
}

template < int DB >
constexpr size_t scatter_smem()
{
   constexpr int D = 1 << DB;
   // staged keys + values (the ranking's per-warp digit words before that),
   // per-warp u16 counters, next global position and output offset per digit,
   // warp totals
   return (size_t)kSortSub * 8 + (size_t)kSortWarps * D * 2 + (size_t)2 * D * 4 + 32 * 4;
}

// One sub-tile of kSortSub items at a time:
//   rank     each warp ranks its 512 items (16 rounds of 32) among the earlier
//            items of the warp with the same digit: a lane ORs its bit into
//            the warp's word of its digit, reads the word back (the lanes of
//            equal digit), and the group's first lane adds the group to the
//            warp's u16 counter of the digit and clears the word;
//   prefix   per digit (DPT consecutive digits per thread): the sub-tile
//            total over the warps, the local start (block scan of the
//            totals), and each warp's first local position of the digit
//            written over its counter;
//   reorder  items to their local positions in shared memory (values read
//            from global memory here, not held through the ranking);
//   write    in local order to global position off[d] + local position:
//            coalesced runs of each digit.
// Two CTAs of 512 threads per SM (104 KB of shared memory, 64 registers each;
// RELM_MP_SORT_THREADS=1024 builds one CTA of 1024 threads per SM with
// 16384-item sub-tiles, faster on uniform keys and slower on skewed ones).
template < int DB >
__global__ void __launch_bounds__(kSortThreads, kSortCtasPerSm) k_sort_scatter(const uint32_t* __restrict__ kin,
                                                                  const int32_t* __restrict__ vin,
                                                                  uint32_t* __restrict__ kout,
                                                                  int32_t* __restrict__ vout, int64_t n, int shift,
                                                                  const int32_t* __restrict__ goff, int64_t ctas,
                                                                  int subs)
{
   constexpr int D = 1 << DB;
   constexpr int DPT = (D + kSortThreads - 1) / kSortThreads;  // digits per thread in the prefix step
   static_assert((size_t)kSortWarps * D * 4 <= (size_t)kSortSub * 8, "digit words must fit in the staging area");
   extern __shared__ __align__(16) unsigned char sm[];
   uint32_t* skey = reinterpret_cast< uint32_t* >(sm);
   int32_t* sval = reinterpret_cast< int32_t* >(skey + kSortSub);
   uint32_t* words = reinterpret_cast< uint32_t* >(sm);  // [warp][digit] lane masks while ranking
   // [warp][digit] counts, then first local positions (16-byte aligned: zeroed with 16-byte stores)
   uint16_t* wh = reinterpret_cast< uint16_t* >(sval + kSortSub);
   int32_t* run = reinterpret_cast< int32_t* >(wh + kSortWarps * D);  // global position of the CTA's next item of digit d
   int32_t* off = run + D;  // this sub-tile: global position of digit d's items minus their local position
   int32_t* wtot = off + D;
   const int tid = threadIdx.x;
   const int lane = tid & 31;
   const int w = tid >> 5;
   const int64_t c = blockIdx.x;
   for(int d = tid; d < D; d += kSortThreads) run[d] = goff[(int64_t)d * ctas + c];
   uint16_t* myh = wh + w * D;
   uint32_t* myw = words + w * D;
   const unsigned lt = lanemask_lt();
   for(int sub = 0; sub < subs; ++sub) {
      const int64_t base = (c * subs + sub) * (int64_t)kSortSub;
      if(base >= n) break;
      const int subn = (n - base) < kSortSub ? (int)(n - base) : kSortSub;
      if(tid == 0) {
         // this sub-tile's values (read at the reorder step) and the next
         // sub-tile's keys
         prefetch_items_l2(vin, base, subn);
         if(sub + 1 < subs && base + kSortSub < n)
            prefetch_items_l2(kin, base + kSortSub, n - base - kSortSub < kSortSub ? n - base - kSortSub : kSortSub);
      }
      for(int i = tid; i < kSortWarps * D / 8; i += kSortThreads)
         reinterpret_cast< uint4* >(wh)[i] = make_uint4(0u, 0u, 0u, 0u);
      for(int i = tid; i < kSortWarps * D / 4; i += kSortThreads)
         reinterpret_cast< uint4* >(words)[i] = make_uint4(0u, 0u, 0u, 0u);
      uint32_t k[kSortPerThread];
#pragma unroll
      for(int r = 0; r < kSortPerThread; ++r) {
         const int idx = w * (kSortSub / kSortWarps) + r * 32 + lane;
         k[r] = idx < subn ? __ldg(kin + base + idx) : 0u;
      }
      __syncthreads();  // counters and digit words zeroed
      uint16_t rank[kSortPerThread];
#pragma unroll
      for(int r = 0; r < kSortPerThread; ++r) {
         const int idx = w * (kSortSub / kSortWarps) + r * 32 + lane;
         const bool valid = idx < subn;
         const unsigned d = (k[r] >> shift) & (D - 1);
         if(valid) atomicOr(&myw[d], 1u << lane);
         __syncwarp();
         const unsigned peers = valid ? myw[d] : 0u;
         __syncwarp();
         const int leader = valid ? __ffs(peers) - 1 : lane;
         int b = 0;
         if(valid && lane == leader) {
            b = myh[d];
            myh[d] = (uint16_t)(b + __popc(peers));
            myw[d] = 0u;
         }
         b = __shfl_sync(0xffffffffu, b, leader);
         rank[r] = (uint16_t)(b + __popc(peers & lt));
         __syncwarp();
      }
      __syncthreads();
      {
         int32_t t[DPT];
         int32_t sum = 0;
#pragma unroll
         for(int j = 0; j < DPT; ++j) {
            const int d = tid * DPT + j;
            int acc = 0;
            if(d < D) {
#pragma unroll
               for(int ww = 0; ww < kSortWarps; ++ww) acc += wh[ww * D + d];
            }
            t[j] = acc;
            sum += acc;
         }
         int32_t total;
         int32_t ex = block_exclusive< SumOp >(sum, wtot, &total);
#pragma unroll
         for(int j = 0; j < DPT; ++j) {
            const int d = tid * DPT + j;
            if(d < D) {
               int acc = ex;
#pragma unroll
               for(int ww = 0; ww < kSortWarps; ++ww) {
                  const int cnt = wh[ww * D + d];
                  wh[ww * D + d] = (uint16_t)acc;
                  acc += cnt;
               }
               const int32_t r0 = run[d];
               off[d] = r0 - ex;
               run[d] = r0 + t[j];
            }
            ex += t[j];
         }
      }
      __syncthreads();
#pragma unroll
      for(int r = 0; r < kSortPerThread; ++r) {
         const int idx = w * (kSortSub / kSortWarps) + r * 32 + lane;
         if(idx < subn) {
            const unsigned d = (k[r] >> shift) & (D - 1);
            const int lp = myh[d] + rank[r];
            skey[lp] = k[r];
            sval[lp] = __ldg(vin + base + idx);
         }
      }
      __syncthreads();
      for(int i = tid; i < subn; i += kSortThreads) {
         const uint32_t key = skey[i];
         const unsigned d = (key >> shift) & (D - 1);
         const int64_t pos = (int64_t)off[d] + i;
         kout[pos] = key;
         vout[pos] = sval[i];
      }
      __syncthreads();  // staging, counters and offsets are rewritten by the next sub-tile
   }
}

template < class Op, bool INCLUSIVE >
int scan_launch(const int32_t* in, int32_t* out, int64_t n, int32_t* part, cudaStream_t stream)
{
   if(n <= 0) return RELM_MP_OK;
   const int64_t nb = scan_blocks(n);
   k_scan_reduce< Op ><<< (unsigned)nb, kScanThreads, 0, stream >>>(in, n, part);
   int rc;
   if((rc = check_launch("k_scan_reduce"))) return rc;
   k_scan_apply< Op, INCLUSIVE ><<< (unsigned)nb, kScanThreads, 0, stream >>>(in, n, part, out);
   return check_launch("k_scan_apply");
}

template < int DB >
int sort_pass(const uint32_t* kin, const int32_t* vin, uint32_t* kout, int32_t* vout, int64_t n, int shift,
              const SortShape& s, int32_t* ghist, int32_t* part, cudaStream_t stream)
{
   constexpr int D = 1 << DB;
   static bool configured = false;  // one attribute call per instantiation (per process)
   if(!configured) {
      const int rc = check_cuda(
         cudaFuncSetAttribute(k_sort_scatter< DB >, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)scatter_smem< DB >()),
         "k_sort_scatter smem attribute"
      );
      if(rc) return rc;
      configured = true;
   }
   int rc;
   k_sort_hist< DB ><<< (unsigned)s.ctas, kSortThreads, 0, stream >>>(kin, n, shift, ghist, s.ctas, s.subs);
   if((rc = check_launch("k_sort_hist"))) return rc;
   if((rc = scan_launch< SumOp, false >(ghist, ghist, (int64_t)D * s.ctas, part, stream))) return rc;
   k_sort_scatter< DB ><<< (unsigned)s.ctas, kSortThreads, scatter_smem< DB >(), stream >>>(
      kin, vin, kout, vout, n, shift, ghist, s.ctas, s.subs
   );
   return check_launch("k_sort_scatter");
}

int sort_pass_bits(int bits, const uint32_t* kin, const int32_t* vin, uint32_t* kout, int32_t* vout, int64_t n,
                   int shift, const SortShape& s, int32_t* ghist, int32_t* part, cudaStream_t stream)
{
   switch(bits) {
      case 1: return sort_pass< 1 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      case 2: return sort_pass< 2 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      case 3: return sort_pass< 3 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      case 4: return sort_pass< 4 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      case 5: return sort_pass< 5 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      case 6: return sort_pass< 6 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      case 7: return sort_pass< 7 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      case 8: return sort_pass< 8 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      case 9: return sort_pass< 9 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      case 10: return sort_pass< 10 >(kin, vin, kout, vout, n, shift, s, ghist, part, stream);
      default: return fail(RELM_MP_ERR_UNSUPPORTED, "radix sort digit width out of range.");
   }
}

}  // namespace

int radix_sort_passes(int end_bit)
{
   const int b = end_bit < 1 ? 1 : end_bit;
   return (b + kSortMaxBits - 1) / kSortMaxBits;
}

size_t radix_sort_temp_bytes(int64_t n, int end_bit)
{
   const SortShape s = sort_shape(n, end_bit);
   int maxbits = 0;
   for(int i = 0; i < s.passes; ++i) maxbits = s.bits[i] > maxbits ? s.bits[i] : maxbits;
   const int64_t counters = ((int64_t)1 << maxbits) * s.ctas;
   return align_up((size_t)counters * 4) + align_up((size_t)scan_blocks(counters) * 4);
}

int radix_sort_pairs(uint32_t* keys, uint32_t* keys_alt, int32_t* vals, int32_t* vals_alt, int64_t n, int end_bit,
                     void* temp, size_t temp_bytes, cudaStream_t stream, bool* in_alt)
{
   *in_alt = false;
   if(n <= 1) return RELM_MP_OK;
   if(temp_bytes < radix_sort_temp_bytes(n, end_bit))
      return fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, "radix sort scratch too small");
   const SortShape s = sort_shape(n, end_bit);
   int maxbits = 0;
   for(int i = 0; i < s.passes; ++i) maxbits = s.bits[i] > maxbits ? s.bits[i] : maxbits;
   const int64_t counters = ((int64_t)1 << maxbits) * s.ctas;
   Carver cv(temp);
   int32_t* ghist = cv.take< int32_t >((size_t)counters);
   int32_t* part = cv.take< int32_t >((size_t)scan_blocks(counters));
   uint32_t* kb[2] = {keys, keys_alt};
   int32_t* vb[2] = {vals, vals_alt};
   int cur = 0;
   for(int i = 0; i < s.passes; ++i) {
      const int rc = sort_pass_bits(s.bits[i], kb[cur], vb[cur], kb[cur ^ 1], vb[cur ^ 1], n, s.shift[i], s, ghist,
                                    part, stream);
      if(rc) return rc;
      cur ^= 1;
   }
   *in_alt = cur == 1;
   return RELM_MP_OK;
}

size_t scan_i32_temp_bytes(int64_t n) { return align_up((size_t)scan_blocks(n) * 4 + 4); }

int scan_max_inclusive(const int32_t* in, int32_t* out, int64_t n, void* temp, size_t temp_bytes,
                       cudaStream_t stream)
{
   if(temp_bytes < scan_i32_temp_bytes(n)) return fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, "scan scratch too small");
   return scan_launch< MaxOp32, true >(in, out, n, static_cast< int32_t* >(temp), stream);
}

}  // namespace relm_mp
