// torch.ops.relm_mp registration of the B200 library.
//
// Registers the reference's schemas (maichmueller/relmo
// src/_ops/mp/mp_ops.cpp:3754-3838) for the hot path and the pack ops its call
// sites use, with:
//   - CUDA kernels for fanout_scatter, fanout_scatter_backward, fanin_reduce,
//     fanin_reduce_sum_backward, fanin_reduce_logsumexp_backward and the four
//     LGAN ops (lgan_pool_reduce, lgan_relation_graph_step and their
//     backwards, sum / mean modes), all running through librelm_mp_b200.so
//     (include/relm_mp.h). There is no CPU or ATen fallback for CUDA tensors:
//     an unsupported dtype raises.
//   - Meta kernels (shapes only) so the ops trace under torch.compile / fake
//     tensors.
//   - CompositeImplicitAutograd pack ops (index arithmetic + cat, as
//     mp_ops.cpp:412-570 and 2511-2773) and build_info.
// CPU tensors go to the CPU kernels of relm_mp_cpu.cpp (the reference
// library's loops and ATen formulas, same results and errors).
//
// Plans (relm_mp_plan) are cached per (output index, gather index) pair. The
// key holds weak references to both index storages plus their version
// counters, offsets, lengths and the bounds, so a freed, reallocated or
// in-place-modified index never hits a stale plan. One model forward reuses
// the same routing indices in every layer and in the backward, so each
// distinct index pair pays the sort once.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/util/intrusive_ptr.h>
#include <torch/library.h>

#include <cmath>
#include <cstdint>
#include <limits>
#include <list>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "relm_mp.h"
#include "relm_mp_torch.h"

#ifndef RELM_MP_BUILD_TORCH_VERSION
#define RELM_MP_BUILD_TORCH_VERSION "unknown"
#endif
#ifndef RELM_MP_BUILD_CUDA_TAG
#define RELM_MP_BUILD_CUDA_TAG "unknown"
#endif
#ifndef RELM_MP_ABI_TARGET
#define RELM_MP_ABI_TARGET "unknown"
#endif

namespace relm_b200 {

using at::Tensor;

constexpr int64_t kModeSum = 0;
constexpr int64_t kModeLogSumExp = 1;

// ---- validation, as mp_ops.cpp:38-71 --------------------------------------

void check_rank(const Tensor& t, int64_t expected, const char* name)
{
   TORCH_CHECK(t.dim() == expected, name, " must be rank ", expected, ", got rank ", t.dim(), ".");
}

void check_int64_index(const Tensor& t, const char* name)
{
   check_rank(t, 1, name);
   TORCH_CHECK(t.scalar_type() == at::kLong, name, " must have dtype torch.int64.");
}

void check_same_device(const Tensor& a, const Tensor& b, const char* an, const char* bn)
{
   TORCH_CHECK(
      a.device() == b.device(), an, " and ", bn, " must be on the same CUDA device, got ", a.device(), " and ",
      b.device(), "."
   );
}

relm_mp_dtype to_dtype(const Tensor& t, const char* op)
{
   switch(t.scalar_type()) {
      case at::kFloat: return RELM_MP_FLOAT32;
      case at::kDouble: return RELM_MP_FLOAT64;
      case at::kBFloat16: return RELM_MP_BFLOAT16;
      case at::kHalf: return RELM_MP_FLOAT16;
      default: break;
   }
   TORCH_CHECK(false, op, ": unsupported dtype ", t.scalar_type(), " (float32, float64, bfloat16, float16).");
   return RELM_MP_FLOAT32;
}

void check_status(int rc, const char* op)
{
   if(rc == RELM_MP_OK) return;
   TORCH_CHECK(false, relm_mp_last_error(), rc == RELM_MP_ERR_INDEX_OUT_OF_RANGE ? "" : " (",
               rc == RELM_MP_ERR_INDEX_OUT_OF_RANGE ? "" : op, rc == RELM_MP_ERR_INDEX_OUT_OF_RANGE ? "" : ")");
}

cudaStream_t stream_of(const Tensor& t)
{
   return at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

Tensor byte_buffer(size_t bytes, const Tensor& like)
{
   return at::empty({(int64_t)std::max< size_t >(bytes, 1)}, like.options().dtype(at::kByte));
}

// ---- plan cache -------------------------------------------------------------

struct IndexKey {
   c10::weak_intrusive_ptr< c10::StorageImpl > storage;
   const c10::StorageImpl* impl = nullptr;
   int64_t offset = 0;
   int64_t numel = 0;
   uint32_t version = 0;

   static IndexKey of(const Tensor& t)
   {
      IndexKey k{c10::weak_intrusive_ptr< c10::StorageImpl >(t.storage().getWeakStorageImpl())};
      k.impl = t.storage().unsafeGetStorageImpl();
      k.offset = t.storage_offset();
      k.numel = t.numel();
      k.version = t.unsafeGetTensorImpl()->version_counter().current_version();
      return k;
   }
   bool alive() const { return !storage.expired(); }
   bool same(const IndexKey& o) const
   {
      return impl == o.impl && offset == o.offset && numel == o.numel && version == o.version;
   }
};

struct PlanEntry {
   IndexKey out_key;
   IndexKey gather_key;
   int64_t num_rows;
   int64_t out_bound;
   int64_t gather_rows;
   int gather_first;
   Tensor memory;  // owns the plan arrays
   relm_mp_plan plan;
   Tensor cover;         // gather-index coverage bitmap (int32 words), computed on first use
   int cover_dups = -1;  // -1 unknown, 0 each gather row at most once, 1 repeats
   bool cover_full = false;  // every gather row is used by some edge (nothing to zero)
   int64_t nonempty_rows = -1;  // output rows holding edges, read on first use
   Tensor gather_counts;        // int32 edges per gathered row, computed on first use
   Tensor host_flags;           // pinned copy of the plan's device flags, filled after the build
   std::shared_ptr< at::cuda::CUDAEvent > flags_copied;  // until the flag bits were learned
   std::shared_ptr< at::cuda::CUDAEvent > flags_event;   // the copy's event (kept for the row count)
   std::shared_ptr< at::cuda::CUDAEvent > ready;  // laid out on a side stream: its end (null: on the user's stream)
};
using PlanPtr = std::shared_ptr< PlanEntry >;

// Working set (bytes of gathered rows in use) above which a copy through a
// destination-ordered plan beats the gather: about 3/4 of the 126 MB L2.
constexpr int64_t kScatterWorkingSet = 96ll << 20;

class PlanCache {
 public:
   static PlanCache& get()
   {
      static PlanCache cache;
      return cache;
   }

   // Returns the plan for (out_index, gather_index); builds it on a miss. With
   // want_cover, a build also computes the gather index's coverage in its
   // validation pass (no separate pass, no extra host sync).
   PlanPtr lookup(const Tensor& out_index, const Tensor& gather_index, int64_t num_rows, int64_t out_bound,
                  int64_t gather_rows, const char* out_name, const char* gather_name, bool gather_first,
                  bool want_cover = false)
   {
      const IndexKey ok = IndexKey::of(out_index);
      const IndexKey gk = IndexKey::of(gather_index);
      {
         std::lock_guard< std::mutex > lock(mu_);
         evict_dead_locked();
         for(auto it = entries_.begin(); it != entries_.end(); ++it) {
            const PlanEntry& e = **it;
            // gather_first only orders the error checks of a build; a cached plan
            // passed both, so fan-out and fan-in over the same pair share it.
            if(e.out_key.same(ok) && e.gather_key.same(gk) && e.num_rows == num_rows && e.out_bound == out_bound
               && e.gather_rows == gather_rows && e.memory.device() == out_index.device()) {
               entries_.splice(entries_.begin(), entries_, it);
               ++hits_;
               learn_flags(*entries_.front());
               wait_ready(entries_.front());
               return entries_.front();
            }
         }
      }
      if(!want_cover)
         if(const PlanPtr t = transposed(out_index, gather_index, out_bound, gather_rows))
            return build_trusted(out_index, gather_index, num_rows, out_bound, gather_rows, t);
      const int64_t num_edges = out_index.numel();
      Tensor memory = byte_buffer(relm_mp_plan_bytes(num_edges, num_rows), out_index);
      relm_mp_plan plan;
      Tensor cover;
      int repeats = -1;
      int64_t covered = -1;
      if(want_cover) {
         Tensor scratch = byte_buffer(relm_mp_plan_cover_scratch_bytes(num_edges, num_rows, gather_rows), out_index);
         cover = at::empty({(int64_t)relm_mp_cover_words(gather_rows)}, out_index.options().dtype(at::kInt));
         const int rc = relm_mp_plan_build_cover(
            out_index.data_ptr< int64_t >(), gather_index.data_ptr< int64_t >(), num_edges, num_rows, out_bound,
            gather_rows, out_name, gather_name, gather_first ? 1 : 0, memory.data_ptr(), (size_t)memory.numel(),
            scratch.data_ptr(), (size_t)scratch.numel(), reinterpret_cast< uint32_t* >(cover.data_ptr< int32_t >()),
            &repeats, &covered, stream_of(out_index), &plan
         );
         check_status(rc, "plan build");
      } else {
         Tensor scratch = byte_buffer(relm_mp_plan_scratch_bytes(num_edges, num_rows), out_index);
         const int rc = relm_mp_plan_build_ex(
            out_index.data_ptr< int64_t >(), gather_index.data_ptr< int64_t >(), num_edges, num_rows, out_bound,
            gather_rows, out_name, gather_name, gather_first ? 1 : 0, memory.data_ptr(), (size_t)memory.numel(),
            scratch.data_ptr(), (size_t)scratch.numel(), stream_of(out_index), &plan
         );
         check_status(rc, "plan build");
      }
      auto entry = std::make_shared< PlanEntry >(
         PlanEntry{ok, gk, num_rows, out_bound, gather_rows, (int)gather_first, memory, plan, cover, repeats,
                   covered == gather_rows, -1, Tensor(), Tensor(), nullptr}
      );
      return insert(entry, out_index);
   }

   // One request of prebuild: the arguments of lookup (no coverage).
   struct Request {
      const Tensor* out_index;
      const Tensor* gather_index;
      int64_t num_rows;
      int64_t out_bound;
      int64_t gather_rows;
      const char* out_name;
      const char* gather_name;
      bool gather_first;
   };

   // Builds the plans of the requests that are not cached yet with one host
   // wait for all of them (relm_mp_plan_build_start / _finish): the index
   // validations run back to back, their results come to the host with one
   // sync, then the layouts are queued. Index errors are raised in request
   // order, so the first failing request gives the error a build of each in
   // turn would have given.
   void prebuild(const std::vector< Request >& reqs)
   {
      struct Pending {
         const Request* r;
         Tensor memory, scratch, stats;
         PlanPtr transposed;  // set: a trusted build (its pair was validated by this plan's build)
      };
      std::vector< Pending > todo;
      for(const Request& r : reqs) {
         if(r.out_index->numel() == 0) continue;
         if(peek(*r.out_index, *r.gather_index, r.num_rows, r.out_bound, r.gather_rows)) continue;
         bool dup = false;  // the same pair twice in one call
         for(const Pending& q : todo)
            if(q.r->out_index->is_same(*r.out_index) && q.r->gather_index->is_same(*r.gather_index) &&
               q.r->num_rows == r.num_rows && q.r->out_bound == r.out_bound && q.r->gather_rows == r.gather_rows)
               dup = true;
         if(dup) continue;
         const int64_t e = r.out_index->numel();
         Pending q{&r, byte_buffer(relm_mp_plan_bytes(e, r.num_rows), *r.out_index),
                   byte_buffer(relm_mp_plan_scratch_bytes(e, r.num_rows), *r.out_index), Tensor(),
                   transposed(*r.out_index, *r.gather_index, r.out_bound, r.gather_rows)};
         if(!q.transposed) {
            q.stats = at::empty({(int64_t)relm_mp_plan_stats_bytes()}, at::TensorOptions().dtype(at::kByte).pinned_memory(true));
         }
         todo.push_back(std::move(q));
      }
      if(todo.empty()) return;
      // The builds run side by side on pool streams, each after the work
      // queued so far on the current stream: a plan of a few million edges
      // fills part of the GPU, one short pass after another. Checked builds
      // validate, the host waits for those streams, then they lay out on the
      // same streams; trusted builds lay out at once. When a build raises, the
      // current stream waits for all of them before anything else is queued on
      // it (the memory and scratch buffers are freed in its order); otherwise
      // each plan's first use waits for its own layout (below).
      const int dev = todo.front().r->out_index->device().index();
      const c10::cuda::CUDAStream main = at::cuda::getCurrentCUDAStream(dev);
      const bool fork = todo.size() > 1;
      std::vector< c10::cuda::CUDAStream > forked;
      auto join = [&]() {
         for(const c10::cuda::CUDAStream& s : forked) {
            at::cuda::CUDAEvent done;
            done.record(s);
            done.block(main);
         }
         forked.clear();
      };
      std::vector< PlanPtr > built(todo.size());
      std::vector< c10::cuda::CUDAStream > on(todo.size(), main);
      try {
         at::cuda::CUDAEvent ready;
         if(fork) ready.record(main);
         for(size_t i = 0; i < todo.size(); ++i) {
            Pending& q = todo[i];
            const Request& r = *q.r;
            const c10::cuda::CUDAStream s = fork ? at::cuda::getStreamFromPool(false, dev) : main;
            if(fork) {
               ready.block(s);
               forked.push_back(s);
            }
            on[i] = s;
            if(q.transposed) {
               built[i] = trusted_entry(*r.out_index, *r.gather_index, r.num_rows, r.out_bound, r.gather_rows,
                                        q.transposed, q.memory, q.scratch, s.stream());
            } else {
               check_status(relm_mp_plan_build_start(
                               r.out_index->data_ptr< int64_t >(), r.gather_index->data_ptr< int64_t >(),
                               r.out_index->numel(), r.num_rows, r.out_bound, r.gather_rows, q.memory.data_ptr(),
                               (size_t)q.memory.numel(), q.scratch.data_ptr(), (size_t)q.scratch.numel(),
                               q.stats.data_ptr(), s.stream()),
                            "plan build");
            }
         }
         for(size_t i = 0; i < todo.size(); ++i) {
            if(todo[i].transposed) continue;
            const cudaError_t err = cudaStreamSynchronize(on[i].stream());
            TORCH_CHECK(err == cudaSuccess, "plan build sync: ", cudaGetErrorString(err));
         }
         for(size_t i = 0; i < todo.size(); ++i) {
            Pending& q = todo[i];
            if(q.transposed) continue;
            const Request& r = *q.r;
            const int64_t e = r.out_index->numel();
            const c10::cuda::CUDAStream s = on[i];
            relm_mp_plan plan;
            check_status(relm_mp_plan_build_finish(
                            r.out_index->data_ptr< int64_t >(), r.gather_index->data_ptr< int64_t >(),
                            e, r.num_rows, r.out_bound, r.gather_rows, r.out_name, r.gather_name,
                            r.gather_first ? 1 : 0, q.memory.data_ptr(), (size_t)q.memory.numel(),
                            q.scratch.data_ptr(), (size_t)q.scratch.numel(), q.stats.data_ptr(), s.stream(), &plan),
                         "plan build");
            built[i] = std::make_shared< PlanEntry >(
               PlanEntry{IndexKey::of(*r.out_index), IndexKey::of(*r.gather_index), r.num_rows,
                         r.out_bound, r.gather_rows, (int)r.gather_first, q.memory, plan, Tensor(), -1, false, -1,
                         Tensor(), Tensor(), nullptr}
            );
         }
      } catch(...) {
         join();  // the memory the builds use is freed in the current stream's order
         throw;
      }
      // No join: each plan carries the end of its layout as an event, which the
      // first use of the plan (a cache hit) puts in front of its kernels, so an
      // op waits for its own plan only and the other layouts run on beside it.
      // The buffers a side stream still uses (the plan memory, its scratch and
      // the two index tensors) are held back from reuse until that stream is
      // past this point.
      for(size_t i = 0; i < built.size(); ++i) {
         const c10::cuda::CUDAStream& s = on[i];
         if(fork) {
            Pending& q = todo[i];
            for(const Tensor* t : std::initializer_list< const Tensor* >{&q.memory, &q.scratch, q.r->out_index,
                                                                          q.r->gather_index})
               c10::cuda::CUDACachingAllocator::recordStream(t->storage().data_ptr(), s);
            built[i]->ready = std::make_shared< at::cuda::CUDAEvent >();
            built[i]->ready->record(s);
         }
         insert(built[i], *todo[i].r->out_index, s);
      }
   }

   // A cached plan of the transposed pair (its output index is this gather
   // index and the other way round) whose bounds are within this pair's: its
   // build validated both indices, so this pair's build need not. Null if
   // there is none. (The LGAN backwards run over the transposes of their
   // forwards' index pairs.)
   PlanPtr transposed(const Tensor& out_index, const Tensor& gather_index, int64_t out_bound, int64_t gather_rows)
   {
      const IndexKey ok = IndexKey::of(out_index);
      const IndexKey gk = IndexKey::of(gather_index);
      std::lock_guard< std::mutex > lock(mu_);
      for(const PlanPtr& e : entries_)
         if(e->out_key.same(gk) && e->gather_key.same(ok) && e->gather_rows <= out_bound &&
            e->out_bound <= gather_rows && e->memory.device() == out_index.device())
            return e;
      return nullptr;
   }

   // The plan entry of a pair that `t`'s build validated, laid out on `stream`
   // into `memory` (relm_mp_plan_bytes) with `scratch`
   // (relm_mp_plan_scratch_bytes, in use until the stream passes this build),
   // without validation and without a host wait: relm_mp_plan_build_identity
   // when t's gather index (this output index) was the identity, else
   // relm_mp_plan_build_trusted (the same sort and layout as a checked build,
   // so the same plan). Not inserted into the cache.
   static PlanPtr trusted_entry(const Tensor& out_index, const Tensor& gather_index, int64_t num_rows,
                                int64_t out_bound, int64_t gather_rows, const PlanPtr& t, const Tensor& memory,
                                const Tensor& scratch, cudaStream_t stream)
   {
      const int64_t e = out_index.numel();
      relm_mp_plan plan;
      const bool identity = (t->plan.flags & RELM_MP_PLAN_GATHER_IDENTITY) && e <= num_rows;
      if(identity) {
         check_status(relm_mp_plan_build_identity(gather_index.data_ptr< int64_t >(), e, num_rows, gather_rows,
                                                  memory.data_ptr(), (size_t)memory.numel(), stream, &plan),
                      "plan build");
      } else {
         check_status(relm_mp_plan_build_trusted(out_index.data_ptr< int64_t >(), gather_index.data_ptr< int64_t >(), e,
                                                 num_rows, gather_rows, memory.data_ptr(), (size_t)memory.numel(),
                                                 scratch.data_ptr(), (size_t)scratch.numel(), stream, &plan),
                      "plan build");
      }
      return std::make_shared< PlanEntry >(
         PlanEntry{IndexKey::of(out_index), IndexKey::of(gather_index), num_rows, out_bound, gather_rows, 0, memory,
                   plan, Tensor(), -1, false, identity ? e : -1, Tensor(), Tensor(), nullptr}
      );
   }

   // trusted_entry on the current stream, cached.
   PlanPtr build_trusted(const Tensor& out_index, const Tensor& gather_index, int64_t num_rows, int64_t out_bound,
                         int64_t gather_rows, const PlanPtr& t)
   {
      const int64_t e = out_index.numel();
      const Tensor memory = byte_buffer(relm_mp_plan_bytes(e, num_rows), out_index);
      const Tensor scratch = byte_buffer(relm_mp_plan_scratch_bytes(e, num_rows), out_index);
      return insert(trusted_entry(out_index, gather_index, num_rows, out_bound, gather_rows, t, memory, scratch,
                                  stream_of(out_index)),
                    out_index);
   }

   // The plan of (flat_src, dst) of a fan-in backward, from the forward's
   // cached plan of (dst, flat_src) when that build found flat_src to be the
   // identity (RELM_MP_PLAN_GATHER_IDENTITY): message row e then holds edge e
   // alone, so the plan is dst as int32 beside row_ptr[r] = min(r, E), built
   // without validation (the forward validated both indices against the same
   // bounds) and without a host wait. Null when that does not apply (the
   // caller then builds the plan the usual way).
   PlanPtr identity_from_forward(const Tensor& src, const Tensor& dst, int64_t num_rows, int64_t out_bound,
                                 int64_t gather_rows, int64_t fwd_gather_rows)
   {
      if(PlanPtr e = peek(src, dst, num_rows, out_bound, gather_rows)) {
         std::lock_guard< std::mutex > lock(mu_);
         ++hits_;
         return e;
      }
      const PlanPtr fp = peek(dst, src, gather_rows, gather_rows, fwd_gather_rows);
      if(!fp || !(fp->plan.flags & RELM_MP_PLAN_GATHER_IDENTITY)) return nullptr;
      const int64_t E = src.numel();
      if(E > out_bound) return nullptr;  // message rows [0, E) must lie in the backward's bound
      Tensor memory = byte_buffer(relm_mp_plan_bytes(E, num_rows), src);
      relm_mp_plan plan;
      check_status(relm_mp_plan_build_identity(dst.data_ptr< int64_t >(), E, num_rows, gather_rows, memory.data_ptr(),
                                               (size_t)memory.numel(), stream_of(src), &plan),
                   "plan build");
      auto entry = std::make_shared< PlanEntry >(
         PlanEntry{IndexKey::of(src), IndexKey::of(dst), num_rows, out_bound, gather_rows, 0, memory, plan, Tensor(), -1,
                   false, E, Tensor(), Tensor(), nullptr}
      );
      return insert(entry, src);
   }

   // The cached plan for the pair, or null (never builds).
   PlanPtr peek(const Tensor& out_index, const Tensor& gather_index, int64_t num_rows, int64_t out_bound,
                int64_t gather_rows)
   {
      const IndexKey ok = IndexKey::of(out_index);
      const IndexKey gk = IndexKey::of(gather_index);
      std::lock_guard< std::mutex > lock(mu_);
      for(const auto& e : entries_)
         if(e->out_key.same(ok) && e->gather_key.same(gk) && e->num_rows == num_rows && e->out_bound == out_bound
            && e->gather_rows == gather_rows && e->memory.device() == out_index.device()) {
            wait_ready(e);
            return e;
         }
      return nullptr;
   }

   // Work queued next on the current stream waits for the entry's layout
   // when that ran on a side stream and has not finished yet (the event is
   // dropped once it has). Under stream capture nothing is queued: event
   // queries are not allowed there, and a plan used in a capture was built
   // by an earlier, uncaptured call.
   static void wait_ready(const PlanPtr& e)
   {
      if(!e->ready) return;
      const c10::cuda::CUDAStream s = at::cuda::getCurrentCUDAStream(e->memory.device().index());
      cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
      if(cudaStreamIsCapturing(s.stream(), &capturing) != cudaSuccess || capturing != cudaStreamCaptureStatusNone)
         return;
      if(e->ready->query()) {
         e->ready.reset();
         return;
      }
      e->ready->block(s);
   }

   // Output rows of the entry's plan that hold edges (read once per plan):
   // from the pinned copy of the plan's device flags made after the build,
   // waiting for that copy only (work queued after the build keeps running).
   int64_t nonempty_rows(const PlanPtr& e, const Tensor& like)
   {
      std::lock_guard< std::mutex > lock(cover_mu_);
      if(e->nonempty_rows < 0) {
         if(e->host_flags.defined() && e->flags_event) {
            e->flags_event->synchronize();
            e->nonempty_rows = e->host_flags.data_ptr< int32_t >()[2];
         } else {
            int64_t rows = 0;
            check_status(relm_mp_plan_nonempty_rows(&e->plan, &rows, stream_of(like)), "plan row count");
            e->nonempty_rows = rows;
         }
      }
      return e->nonempty_rows;
   }

   // Coverage of the entry's gather index (computed once per plan; a plan
   // built with want_cover has it already).
   void ensure_cover(const PlanPtr& e, const Tensor& like)
   {
      std::lock_guard< std::mutex > lock(cover_mu_);
      if(e->cover_dups >= 0) return;
      Tensor cover = at::empty({(int64_t)relm_mp_cover_words(e->gather_rows)}, like.options().dtype(at::kInt));
      Tensor scratch = byte_buffer(relm_mp_plan_gather_cover_scratch_bytes(&e->plan), like);
      int dups = 0;
      int64_t covered = -1;
      check_status(relm_mp_plan_gather_cover_ex(&e->plan, reinterpret_cast< uint32_t* >(cover.data_ptr< int32_t >()),
                                                &dups, &covered, scratch.data_ptr(), (size_t)scratch.numel(),
                                                stream_of(like)),
                   "gather cover");
      e->cover = cover;
      e->cover_dups = dups;
      e->cover_full = covered == e->gather_rows;
   }

   // Edges per gathered row of the entry's plan (computed once per plan).
   const int32_t* gather_counts(const PlanPtr& e, const Tensor& like)
   {
      std::lock_guard< std::mutex > lock(cover_mu_);
      if(!e->gather_counts.defined()) {
         Tensor counts = at::empty({std::max< int64_t >(e->gather_rows, 1)}, like.options().dtype(at::kInt));
         check_status(relm_mp_plan_gather_counts(&e->plan, counts.data_ptr< int32_t >(), stream_of(like)),
                      "gather counts");
         e->gather_counts = counts;
      }
      return e->gather_counts.data_ptr< int32_t >();
   }

   void clear()
   {
      std::lock_guard< std::mutex > lock(mu_);
      entries_.clear();
   }

   std::vector< int64_t > stats()
   {
      std::lock_guard< std::mutex > lock(mu_);
      evict_dead_locked();
      int64_t bytes = 0;
      for(const auto& e : entries_)
         bytes += e->memory.numel() + (e->cover.defined() ? e->cover.numel() * 4 : 0) +
                  (e->gather_counts.defined() ? e->gather_counts.numel() * 4 : 0);
      return {(int64_t)entries_.size(), hits_, builds_, bytes, (int64_t)capacity_};
   }

   void set_capacity(int64_t cap)
   {
      std::lock_guard< std::mutex > lock(mu_);
      capacity_ = (size_t)std::max< int64_t >(cap, 0);
      while(entries_.size() > capacity_) entries_.pop_back();
   }

 private:
   // Sets the plan's host flag bits once the copy of its device flags landed.
   // Adds a built plan: queues the copy of its device flags to pinned host
   // memory (no sync; once it has landed, later calls launch only the kernels
   // the plan needs) and puts the entry at the front of the cache.
   // Caches the entry; its flags are copied to the host on the stream that
   // built it (the current stream unless given).
   PlanPtr insert(const PlanPtr& entry, const Tensor& like, const c10::optional< c10::cuda::CUDAStream >& built_on = {})
   {
      entry->host_flags = at::empty({4}, at::TensorOptions().dtype(at::kInt).pinned_memory(true));
      const c10::cuda::CUDAStream cs = built_on ? *built_on : at::cuda::getCurrentCUDAStream(like.device().index());
      const cudaError_t err = cudaMemcpyAsync(entry->host_flags.data_ptr(), entry->plan.device_flags,
                                              4 * sizeof(int32_t), cudaMemcpyDeviceToHost, cs.stream());
      TORCH_CHECK(err == cudaSuccess, "plan flags copy: ", cudaGetErrorString(err));
      entry->flags_copied = std::make_shared< at::cuda::CUDAEvent >();
      entry->flags_copied->record(cs);
      entry->flags_event = entry->flags_copied;
      std::lock_guard< std::mutex > lock(mu_);
      ++builds_;
      entries_.push_front(entry);
      while(entries_.size() > capacity_) entries_.pop_back();
      return entry;
   }

   static void learn_flags(PlanEntry& e)
   {
      if((e.plan.flags & RELM_MP_PLAN_FLAGS_KNOWN) || !e.flags_copied || !e.flags_copied->query()) return;
      const int32_t* f = e.host_flags.data_ptr< int32_t >();
      e.plan.flags |= RELM_MP_PLAN_FLAGS_KNOWN | (f[0] ? RELM_MP_PLAN_REPEATS : 0u) | (f[1] ? RELM_MP_PLAN_LONG_ROWS : 0u);
      e.flags_copied.reset();
   }

   void evict_dead_locked()
   {
      for(auto it = entries_.begin(); it != entries_.end();) {
         if(!(*it)->out_key.alive() || !(*it)->gather_key.alive())
            it = entries_.erase(it);
         else
            ++it;
      }
   }

   std::mutex mu_;
   std::mutex cover_mu_;
   std::list< PlanPtr > entries_;
   size_t capacity_ = 16;
   int64_t hits_ = 0;
   int64_t builds_ = 0;
};

// The coverage bitmap of the entry's gather index for the scatter kernels, or
// null when every gather row is covered (they then zero nothing).
const uint32_t* cover_bits(const PlanPtr& e)
{
   if(e->cover_full) return nullptr;
   return reinterpret_cast< const uint32_t* >(e->cover.data_ptr< int32_t >());
}

relm_mp_plan get_plan(const Tensor& out_index, const Tensor& gather_index, int64_t num_rows, int64_t out_bound,
                      int64_t gather_rows, const char* out_name, const char* gather_name, bool gather_first,
                      Tensor* keep_alive)
{
   const PlanPtr e = PlanCache::get().lookup(
      out_index, gather_index, num_rows, out_bound, gather_rows, out_name, gather_name, gather_first
   );
   *keep_alive = e->memory;
   return e->plan;
}

Tensor contig(const Tensor& t) { return t.is_contiguous() ? t : t.contiguous(); }

// ---- CUDA kernels of the hot ops ------------------------------------------------

// mp_ops.cpp:3038-3101
Tensor fanout_scatter_cuda(const Tensor& x_cat, const Tensor& src_global_idx, const Tensor& flat_dst, int64_t out_rows)
{
   check_rank(x_cat, 2, "x_cat");
   check_int64_index(src_global_idx, "src_global_idx");
   check_int64_index(flat_dst, "flat_dst");
   TORCH_CHECK(src_global_idx.size(0) == flat_dst.size(0), "src_global_idx and flat_dst must have equal length.");
   TORCH_CHECK(out_rows >= 0, "out_rows must be >= 0.");
   check_same_device(x_cat, src_global_idx, "x_cat", "src_global_idx");
   check_same_device(x_cat, flat_dst, "x_cat", "flat_dst");
   c10::cuda::CUDAGuard guard(x_cat.device());
   const relm_mp_dtype dt = to_dtype(x_cat, "fanout_scatter");
   const int64_t emb = x_cat.size(1);
   if(src_global_idx.numel() == 0 || out_rows == 0) return at::zeros({out_rows, emb}, x_cat.options());
   Tensor out = at::empty({out_rows, emb}, x_cat.options());
   const Tensor x = contig(x_cat);
   const Tensor src = contig(src_global_idx);
   const Tensor dst = contig(flat_dst);
   // Source plan (shared with fanout_scatter_backward): each x row is read once
   // and stored into its slots, when every slot is written at most once.
   const PlanPtr sp = PlanCache::get().lookup(
      src, dst, x.size(0), x.size(0), out_rows, "src_global_idx", "flat_dst", false, /*want_cover=*/true
   );
   PlanCache::get().ensure_cover(sp, x);
   if(sp->cover_dups == 0) {
      check_status(relm_mp_plan_scatter_rows(&sp->plan, dt, x.data_ptr(), emb, cover_bits(sp),
                                             out.data_ptr(), stream_of(x)),
                   "fanout_scatter");
      return out;
   }
   // Repeated slots: order by slot, the highest edge of each slot wins.
   Tensor keep;
   const relm_mp_plan plan = get_plan(dst, src, out_rows, out_rows, x.size(0), "flat_dst", "src_global_idx", true, &keep);
   check_status(relm_mp_plan_gather_last(&plan, dt, x.data_ptr(), emb, out.data_ptr(), stream_of(x)), "fanout_scatter");
   return out;
}

Tensor planned_sum(const relm_mp_plan& plan, relm_mp_dtype dt, const Tensor& table, int64_t emb, Tensor& out,
                   int mode, const char* op, const relm_mp_lse_form* form = nullptr)
{
   Tensor scratch = byte_buffer(relm_mp_plan_reduce_scratch_bytes(&plan, emb, dt, mode), table);
   const int rc = form ? relm_mp_plan_reduce_lse(&plan, dt, form, table.data_ptr(), emb, out.data_ptr(),
                                                 scratch.data_ptr(), (size_t)scratch.numel(), stream_of(table))
                       : relm_mp_plan_reduce(&plan, dt, mode, table.data_ptr(), emb, out.data_ptr(),
                                             scratch.data_ptr(), (size_t)scratch.numel(), stream_of(table));
   check_status(rc, op);
   return out;
}

// mp_ops.cpp:3103-3166
Tensor fanout_scatter_backward_cuda(const Tensor& grad_out, const Tensor& src_global_idx, const Tensor& flat_dst,
                                    int64_t x_rows)
{
   check_rank(grad_out, 2, "grad_out");
   check_int64_index(src_global_idx, "src_global_idx");
   check_int64_index(flat_dst, "flat_dst");
   TORCH_CHECK(src_global_idx.size(0) == flat_dst.size(0), "src_global_idx and flat_dst must have equal length.");
   TORCH_CHECK(x_rows >= 0, "x_rows must be >= 0.");
   check_same_device(grad_out, src_global_idx, "grad_out", "src_global_idx");
   check_same_device(grad_out, flat_dst, "grad_out", "flat_dst");
   c10::cuda::CUDAGuard guard(grad_out.device());
   const relm_mp_dtype dt = to_dtype(grad_out, "fanout_scatter_backward");
   const int64_t emb = grad_out.size(1);
   if(src_global_idx.numel() == 0 || x_rows == 0) return at::zeros({x_rows, emb}, grad_out.options());
   Tensor grad_x = at::empty({x_rows, emb}, grad_out.options());
   const Tensor g = contig(grad_out);
   const Tensor src = contig(src_global_idx);
   const Tensor dst = contig(flat_dst);
   Tensor keep;
   const relm_mp_plan plan = get_plan(src, dst, x_rows, x_rows, g.size(0), "src_global_idx", "flat_dst", false, &keep);
   return planned_sum(plan, dt, g, emb, grad_x, RELM_MP_MODE_SUM, "fanout_scatter_backward");
}

// Value of rows without messages: 0 (sum), -inf (plain logsumexp) or
// (1/beta) log(eps) (smoothed; computed in the accumulator type).
double empty_row_value(int64_t mode, const relm_mp_lse_form* form, const Tensor& like)
{
   if(mode == kModeSum) return 0.0;
   if(!form) return -std::numeric_limits< double >::infinity();
   if(like.scalar_type() == at::kDouble) return (1.0 / form->beta) * std::log(form->eps);
   return (double)((1.0f / (float)form->beta) * std::log((float)form->eps));
}

Tensor fanin_reduce_cuda_impl(const Tensor& rel_flat, const Tensor& flat_src, const Tensor& dst_idx, int64_t dim_size,
                              int64_t mode, const relm_mp_lse_form* form);

// mp_ops.cpp:3327-3348 with 3168-3222 (sum) and 3005-3036 (logsumexp)
Tensor fanin_reduce_cuda(const Tensor& rel_flat, const Tensor& flat_src, const Tensor& dst_idx, int64_t dim_size,
                         int64_t mode)
{
   return fanin_reduce_cuda_impl(rel_flat, flat_src, dst_idx, dim_size, mode, nullptr);
}

Tensor fanin_reduce_cuda_impl(const Tensor& rel_flat, const Tensor& flat_src, const Tensor& dst_idx, int64_t dim_size,
                              int64_t mode, const relm_mp_lse_form* form)
{
   check_rank(rel_flat, 2, "rel_flat");
   check_int64_index(flat_src, "flat_src");
   check_int64_index(dst_idx, "dst_idx");
   TORCH_CHECK(flat_src.size(0) == dst_idx.size(0), "flat_src and dst_idx must have equal length.");
   TORCH_CHECK(dim_size >= 0, "dim_size must be >= 0.");
   if(mode != kModeSum && mode != kModeLogSumExp)
      throw std::invalid_argument("Unsupported fanin_reduce mode. Supported: 0=sum, 1=logsumexp.");
   check_same_device(rel_flat, flat_src, "rel_flat", "flat_src");
   check_same_device(rel_flat, dst_idx, "rel_flat", "dst_idx");
   c10::cuda::CUDAGuard guard(rel_flat.device());
   const relm_mp_dtype dt = to_dtype(rel_flat, "fanin_reduce");
   const int64_t emb = rel_flat.size(1);
   if(flat_src.numel() == 0 || dim_size == 0) {
      if(mode == kModeSum) return at::zeros({dim_size, emb}, rel_flat.options());
      return at::full({dim_size, emb}, empty_row_value(mode, form, rel_flat), rel_flat.options());
   }
   Tensor out = at::empty({dim_size, emb}, rel_flat.options());
   const Tensor rel = contig(rel_flat);
   const Tensor src = contig(flat_src);
   const Tensor dst = contig(dst_idx);
   Tensor keep;
   const relm_mp_plan plan = get_plan(dst, src, dim_size, dim_size, rel.size(0), "dst_idx", "flat_src", true, &keep);
   return planned_sum(plan, dt, rel, emb, out, (int)mode, "fanin_reduce", mode == kModeLogSumExp ? form : nullptr);
}

// mp_ops.cpp:3224-3284
Tensor fanin_reduce_sum_backward_cuda(const Tensor& grad_out, const Tensor& flat_src, const Tensor& dst_idx,
                                      int64_t rel_rows)
{
   check_rank(grad_out, 2, "grad_out");
   check_int64_index(flat_src, "flat_src");
   check_int64_index(dst_idx, "dst_idx");
   TORCH_CHECK(flat_src.size(0) == dst_idx.size(0), "flat_src and dst_idx must have equal length.");
   TORCH_CHECK(rel_rows >= 0, "rel_rows must be >= 0.");
   check_same_device(grad_out, flat_src, "grad_out", "flat_src");
   check_same_device(grad_out, dst_idx, "grad_out", "dst_idx");
   c10::cuda::CUDAGuard guard(grad_out.device());
   const relm_mp_dtype dt = to_dtype(grad_out, "fanin_reduce_sum_backward");
   const int64_t emb = grad_out.size(1);
   if(flat_src.numel() == 0 || rel_rows == 0) return at::zeros({rel_rows, emb}, grad_out.options());
   Tensor grad_rel = at::empty({rel_rows, emb}, grad_out.options());
   const Tensor g = contig(grad_out);
   const Tensor src = contig(flat_src);
   const Tensor dst = contig(dst_idx);
   // With flat_src repeating no row, grad_rel rows are copies of grad_out rows.
   // When the grad_out rows in use outgrow L2, each is read once in destination
   // order through the forward's plan and stored to its message rows (no
   // re-reads from HBM); below that the per-message-row gather is faster.
   const int64_t row_bytes = emb * (int64_t)g.element_size();
   if(g.size(0) * row_bytes > kScatterWorkingSet) {
      PlanCache& cache = PlanCache::get();
      if(const PlanPtr fp = cache.peek(dst, src, g.size(0), g.size(0), rel_rows)) {
         if(cache.nonempty_rows(fp, g) * row_bytes > kScatterWorkingSet) {
            cache.ensure_cover(fp, g);
            if(fp->cover_dups == 0) {
               check_status(relm_mp_plan_scatter_rows(&fp->plan, dt, g.data_ptr(), emb,
                                                      cover_bits(fp), grad_rel.data_ptr(),
                                                      stream_of(g)),
                            "fanin_reduce_sum_backward");
               return grad_rel;
            }
         }
      }
   }
   Tensor keep;
   relm_mp_plan plan;
   if(const PlanPtr ip = PlanCache::get().identity_from_forward(src, dst, rel_rows, rel_rows, g.size(0), rel_rows)) {
      keep = ip->memory;
      plan = ip->plan;
   } else {
      plan = get_plan(src, dst, rel_rows, rel_rows, g.size(0), "flat_src", "dst_idx", false, &keep);
   }
   return planned_sum(plan, dt, g, emb, grad_rel, RELM_MP_MODE_SUM, "fanin_reduce_sum_backward");
}

Tensor lse_backward_cuda_impl(const Tensor& grad_out, const Tensor& rel_flat, const Tensor& flat_src,
                              const Tensor& dst_idx, const Tensor& out, int64_t rel_rows,
                              const relm_mp_lse_form* form);

// mp_ops.cpp:3286-3325
Tensor fanin_reduce_logsumexp_backward_cuda(const Tensor& grad_out, const Tensor& rel_flat, const Tensor& flat_src,
                                            const Tensor& dst_idx, const Tensor& out, int64_t rel_rows)
{
   return lse_backward_cuda_impl(grad_out, rel_flat, flat_src, dst_idx, out, rel_rows, nullptr);
}

Tensor lse_backward_cuda_impl(const Tensor& grad_out, const Tensor& rel_flat, const Tensor& flat_src,
                              const Tensor& dst_idx, const Tensor& out, int64_t rel_rows,
                              const relm_mp_lse_form* form)
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
   check_same_device(grad_out, rel_flat, "grad_out", "rel_flat");
   check_same_device(grad_out, flat_src, "grad_out", "flat_src");
   check_same_device(grad_out, dst_idx, "grad_out", "dst_idx");
   check_same_device(grad_out, out, "grad_out", "out");
   TORCH_CHECK(
      grad_out.scalar_type() == rel_flat.scalar_type() && grad_out.scalar_type() == out.scalar_type(),
      "grad_out, rel_flat, and out must share dtype."
   );
   c10::cuda::CUDAGuard guard(grad_out.device());
   const relm_mp_dtype dt = to_dtype(grad_out, "fanin_reduce_logsumexp_backward");
   const int64_t emb = grad_out.size(1);
   if(flat_src.numel() == 0 || rel_rows == 0) return at::zeros({rel_rows, emb}, rel_flat.options());
   Tensor grad_rel = at::empty({rel_rows, emb}, rel_flat.options());
   const Tensor g = contig(grad_out);
   const Tensor rel = contig(rel_flat);
   const Tensor o = contig(out);
   const Tensor src = contig(flat_src);
   const Tensor dst = contig(dst_idx);
   // As in the sum backward: with flat_src repeating no row and the grad_out /
   // out rows in use above the L2 working set, walk the forward's plan in
   // destination order, reading each destination's grad_out and out rows once.
   const int64_t row_bytes = emb * (int64_t)g.element_size();
   if(g.size(0) * row_bytes > kScatterWorkingSet && rel.size(0) == rel_rows) {
      PlanCache& cache = PlanCache::get();
      if(const PlanPtr fp = cache.peek(dst, src, g.size(0), g.size(0), rel_rows)) {
         if(cache.nonempty_rows(fp, g) * row_bytes > kScatterWorkingSet) {
            cache.ensure_cover(fp, g);
            if(fp->cover_dups == 0) {
               const int rc = relm_mp_plan_scatter_logsumexp_backward_ex(
                  &fp->plan, dt, form, g.data_ptr(), o.data_ptr(), rel.data_ptr(), emb, cover_bits(fp),
                  grad_rel.data_ptr(), stream_of(g)
               );
               if(rc != RELM_MP_ERR_UNSUPPORTED) {  // unsupported row shape: the per-message-row path below
                  check_status(rc, "fanin_reduce_logsumexp_backward");
                  return grad_rel;
               }
            }
         }
      }
   }
   Tensor keep;
   const int64_t bound = std::min(rel_rows, rel.size(0));
   relm_mp_plan plan;
   if(const PlanPtr ip = PlanCache::get().identity_from_forward(src, dst, rel_rows, bound, g.size(0), rel.size(0))) {
      keep = ip->memory;
      plan = ip->plan;
   } else {
      plan = get_plan(src, dst, rel_rows, bound, g.size(0), "flat_src", "dst_idx", false, &keep);
   }
   Tensor scratch = byte_buffer(relm_mp_plan_reduce_scratch_bytes(&plan, emb, dt, RELM_MP_MODE_LOGSUMEXP_BACKWARD), g);
   check_status(
      relm_mp_plan_logsumexp_backward_ex(&plan, dt, form, g.data_ptr(), o.data_ptr(), rel.data_ptr(), emb,
                                         grad_rel.data_ptr(), scratch.data_ptr(), (size_t)scratch.numel(),
                                         stream_of(g)),
      "fanin_reduce_logsumexp_backward"
   );
   return grad_rel;
}

// ---- smoothed logsumexp (relmo's LogSumExpAggregation, models/aggr.py:96-123) ------------
//
// The aggregation relmo's models use for "logsumexp": per column,
// m + (1/beta) log(eps + sum e^(beta (x - m))) with m the row max (no gradient
// through it), (1/beta) log(eps) for rows without messages. Same arguments
// and checks as fanin_reduce / fanin_reduce_logsumexp_backward, plus beta and
// eps; the backward weight is e^(beta (x - out)). Not part of the reference's
// op library (relmo computes it with ATen around index_reduce_).

relm_mp_lse_form smoothed_form(double beta, double eps)
{
   TORCH_CHECK(beta > 0.0 && std::isfinite(beta), "smoothed logsumexp needs a finite beta > 0.");
   TORCH_CHECK(eps >= 0.0, "smoothed logsumexp needs eps >= 0.");
   return relm_mp_lse_form{beta, eps};
}

Tensor smoothed_logsumexp_cuda(const Tensor& rel_flat, const Tensor& flat_src, const Tensor& dst_idx, int64_t dim_size,
                               double beta, double eps)
{
   const relm_mp_lse_form f = smoothed_form(beta, eps);
   return fanin_reduce_cuda_impl(rel_flat, flat_src, dst_idx, dim_size, kModeLogSumExp, &f);
}

Tensor smoothed_logsumexp_backward_cuda(const Tensor& grad_out, const Tensor& rel_flat, const Tensor& flat_src,
                                        const Tensor& dst_idx, const Tensor& out, int64_t rel_rows, double beta)
{
   const relm_mp_lse_form f = smoothed_form(beta, 0.0);
   return lse_backward_cuda_impl(grad_out, rel_flat, flat_src, dst_idx, out, rel_rows, &f);
}

Tensor smoothed_logsumexp_meta(const Tensor& rel_flat, const Tensor&, const Tensor&, int64_t dim_size, double, double)
{
   return at::empty({dim_size, rel_flat.size(1)}, rel_flat.options());
}

Tensor smoothed_logsumexp_backward_meta(const Tensor&, const Tensor& rel_flat, const Tensor&, const Tensor&,
                                        const Tensor&, int64_t rel_rows, double)
{
   return at::empty({rel_rows, rel_flat.size(1)}, rel_flat.options());
}

// ---- Meta (shape) kernels ------------------------------------------------------

Tensor fanout_scatter_meta(const Tensor& x_cat, const Tensor&, const Tensor&, int64_t out_rows)
{
   return at::empty({out_rows, x_cat.size(1)}, x_cat.options());
}
Tensor fanout_scatter_backward_meta(const Tensor& grad_out, const Tensor&, const Tensor&, int64_t x_rows)
{
   return at::empty({x_rows, grad_out.size(1)}, grad_out.options());
}
Tensor fanin_reduce_meta(const Tensor& rel_flat, const Tensor&, const Tensor&, int64_t dim_size, int64_t)
{
   return at::empty({dim_size, rel_flat.size(1)}, rel_flat.options());
}
Tensor fanin_reduce_sum_backward_meta(const Tensor& grad_out, const Tensor&, const Tensor&, int64_t rel_rows)
{
   return at::empty({rel_rows, grad_out.size(1)}, grad_out.options());
}
Tensor fanin_reduce_logsumexp_backward_meta(const Tensor& grad_out, const Tensor& rel_flat, const Tensor&,
                                            const Tensor&, const Tensor&, int64_t rel_rows)
{
   return at::empty({rel_rows, grad_out.size(1)}, rel_flat.options());
}

// ---- pack ops (index arithmetic; mp_ops.cpp:412-570, 2511-2773) ------------------

Tensor cat_or_single(const std::vector< Tensor >& parts)
{
   return parts.size() == 1 ? parts[0] : at::cat(parts, 0);
}

Tensor empty_index_like(const Tensor& ref) { return at::empty({0}, ref.options().dtype(at::kLong)); }

// The index arithmetic of a pack op, part k: idx_k * mul_k + add_k, concatenated.
// CUDA index parts on one device: one relm_mp_pack_index launch (per 64
// parts); otherwise the ATen formula (a kernel per part plus a cat).
bool all_on_one_cuda_device(const std::vector< Tensor >& parts)
{
   if(parts.empty() || !parts[0].is_cuda()) return false;
   for(const auto& t : parts)
      if(!t.is_cuda() || t.device() != parts[0].device()) return false;
   return true;
}

Tensor pack_index(const std::vector< Tensor >& parts, const std::vector< int64_t >& mul,
                  const std::vector< int64_t >& add, const Tensor& like)
{
   if(parts.empty()) return empty_index_like(like);
   if(parts.size() == 1 && mul[0] == 1 && add[0] == 0) return parts[0];
   if(!all_on_one_cuda_device(parts)) {
      std::vector< Tensor > terms;
      for(size_t i = 0; i < parts.size(); ++i)
         terms.push_back(mul[i] == 1 ? parts[i] + add[i] : parts[i] * mul[i] + add[i]);
      return cat_or_single(terms);
   }
   c10::cuda::CUDAGuard guard(parts[0].device());
   int64_t total = 0;
   std::vector< Tensor > keep;
   std::vector< relm_mp_index_part > ps;
   for(size_t i = 0; i < parts.size(); ++i) {
      keep.push_back(contig(parts[i]));
      ps.push_back(relm_mp_index_part{keep.back().data_ptr< int64_t >(), keep.back().numel(), mul[i], add[i]});
      total += keep.back().numel();
   }
   Tensor out = at::empty({total}, parts[0].options());
   check_status(relm_mp_pack_index(ps.data(), (int)ps.size(), out.data_ptr< int64_t >(), stream_of(parts[0])),
                "pack index");
   return out;
}

// The argument checks of the pack ops follow the reference's order and
// messages (mp_ops.cpp:412-570, 2511-2773): callers match on them.

// Rank, device, dtype and embedding dim of every value part (`vname` is
// "x_parts" or "rel_parts").
void check_value_parts(const std::vector< Tensor >& parts, const char* op, const char* vname)
{
   const std::string first = std::string(vname) + "[0]";
   const std::string each = std::string(vname) + "[i]";
   check_rank(parts[0], 2, first.c_str());
   for(size_t i = 0; i < parts.size(); ++i) {
      const Tensor& v = parts[i];
      check_rank(v, 2, each.c_str());
      TORCH_CHECK(v.device() == parts[0].device(), op, " expects all ", vname, " on the same device. Mismatch at part ",
                  i, ".");
      TORCH_CHECK(v.scalar_type() == parts[0].scalar_type(), op, " expects all ", vname,
                  " with the same dtype. Mismatch at part ", i, ".");
      TORCH_CHECK(v.size(1) == parts[0].size(1), op, " expects matching embedding dim across ", vname, ". Part ", i,
                  " has emb=", v.size(1), ", expected ", parts[0].size(1), ".");
   }
}

// fanout_pack_multi / fanin_pack_multi (mp_ops.cpp:412-570): the value parts
// concatenated, the first index of part k offset by the rows of parts < k,
// the second index concatenated.
std::tuple< Tensor, Tensor, Tensor > pack_multi(const std::vector< Tensor >& value_parts,
                                                const std::vector< Tensor >& first_idx_parts,
                                                const std::vector< Tensor >& second_idx_parts, const char* op,
                                                const char* what, const char* vname, const char* first_name,
                                                const char* second_name)
{
   TORCH_CHECK(!value_parts.empty(), op, " requires at least one ", what, ".");
   TORCH_CHECK(value_parts.size() == first_idx_parts.size() && value_parts.size() == second_idx_parts.size(), op,
               " expects ", vname, ", ", first_name, "_parts, and ", second_name, "_parts with equal lengths.");
   const std::string first_each = std::string(first_name) + "_parts[i]";
   const std::string second_each = std::string(second_name) + "_parts[i]";
   const std::string vfirst = std::string(vname) + "[0]";
   const std::string veach = std::string(vname) + "[i]";
   check_rank(value_parts[0], 2, vfirst.c_str());
   std::vector< int64_t > first_add;
   int64_t offset = 0;
   for(size_t i = 0; i < value_parts.size(); ++i) {
      const Tensor& v = value_parts[i];
      check_rank(v, 2, veach.c_str());
      check_int64_index(first_idx_parts[i], first_each.c_str());
      check_int64_index(second_idx_parts[i], second_each.c_str());
      TORCH_CHECK(v.device() == value_parts[0].device(), op, " expects all ", vname,
                  " on the same device. Mismatch at part ", i, ".");
      TORCH_CHECK(v.scalar_type() == value_parts[0].scalar_type(), op, " expects all ", vname,
                  " with the same dtype. Mismatch at part ", i, ".");
      TORCH_CHECK(v.size(1) == value_parts[0].size(1), op, " expects matching embedding dim across ", vname, ". Part ",
                  i, " has emb=", v.size(1), ", expected ", value_parts[0].size(1), ".");
      TORCH_CHECK(first_idx_parts[i].device() == value_parts[0].device() &&
                     second_idx_parts[i].device() == value_parts[0].device(),
                  op, " expects all index tensors on the same device as ", vname, ".");
      TORCH_CHECK(first_idx_parts[i].size(0) == second_idx_parts[i].size(0), op, " expects ", first_name, " and ",
                  second_name, " lengths to match for part ", i, ".");
      first_add.push_back(offset);
      offset += v.size(0);
   }
   const std::vector< int64_t > ones(value_parts.size(), 1), zeros(value_parts.size(), 0);
   return {cat_or_single(value_parts), pack_index(first_idx_parts, ones, first_add, value_parts[0]),
           pack_index(second_idx_parts, ones, zeros, value_parts[0])};
}

std::tuple< Tensor, Tensor, Tensor > fanout_pack_multi(at::TensorList x_parts, at::TensorList src_idx_parts,
                                                       at::TensorList flat_dst_parts)
{
   return pack_multi(x_parts.vec(), src_idx_parts.vec(), flat_dst_parts.vec(), "fanout_pack_multi", "source tensor",
                     "x_parts", "src_idx", "flat_dst");
}

std::tuple< Tensor, Tensor, Tensor > fanin_pack_multi(at::TensorList rel_parts, at::TensorList flat_src_parts,
                                                      at::TensorList dst_idx_parts)
{
   return pack_multi(rel_parts.vec(), flat_src_parts.vec(), dst_idx_parts.vec(), "fanin_pack_multi",
                     "relation tensor", "rel_parts", "flat_src", "dst_idx");
}

// Checks of one edge part of the *_pack_from_edges ops; returns its value part.
int64_t check_edge_part(const Tensor& src, const Tensor& dst, const Tensor& ref, size_t i, int64_t part,
                        size_t num_values, const char* op, const char* vname, const char* part_ids)
{
   check_int64_index(src, "edge_src_parts[i]");
   check_int64_index(dst, "edge_dst_parts[i]");
   TORCH_CHECK(src.device() == ref.device() && dst.device() == ref.device(), op,
               " expects all edge index tensors on the same device as ", vname, ".");
   TORCH_CHECK(src.size(0) == dst.size(0), op, " expects edge src/dst lengths to match for part ", i, ".");
   TORCH_CHECK(part >= 0 && part < (int64_t)num_values, op, " ", part_ids, "[", i, "] out of range: ", part, ".");
   return part;
}

// fanout_pack_from_edges (mp_ops.cpp:2511-2614): edge part k gathers rows
// src_k of value part p_k (offset by the rows before it) into slots
// slot_offset_k + dst_k * arity_k + pos_k.
std::tuple< Tensor, Tensor, Tensor > fanout_pack_from_edges(at::TensorList x_parts, at::TensorList edge_src_parts,
                                                            at::TensorList edge_dst_parts, at::IntArrayRef src_part_ids,
                                                            at::IntArrayRef arity_parts, at::IntArrayRef pos_parts,
                                                            at::IntArrayRef slot_offset_parts)
{
   const char* op = "fanout_pack_from_edges";
   TORCH_CHECK(!x_parts.empty(), op, " requires at least one source tensor.");
   const size_t n = edge_src_parts.size();
   TORCH_CHECK(edge_dst_parts.size() == n, op, " expects edge_src_parts and edge_dst_parts with equal lengths.");
   TORCH_CHECK(src_part_ids.size() == n && arity_parts.size() == n && pos_parts.size() == n &&
                  slot_offset_parts.size() == n,
               op, " expects metadata arrays to match number of edge parts.");
   const std::vector< Tensor > xs = x_parts.vec();
   check_value_parts(xs, op, "x_parts");
   std::vector< int64_t > offsets;
   int64_t offset = 0;
   for(const auto& x : xs) {
      offsets.push_back(offset);
      offset += x.size(0);
   }
   const Tensor x_cat = cat_or_single(xs);
   if(n == 0) return {x_cat, empty_index_like(xs[0]), empty_index_like(xs[0])};
   std::vector< Tensor > srcs, dsts;
   std::vector< int64_t > src_mul, src_add, dst_mul, dst_add;
   for(size_t i = 0; i < n; ++i) {
      const int64_t part = check_edge_part(edge_src_parts[i], edge_dst_parts[i], xs[0], i, src_part_ids[i],
                                           xs.size(), op, "x_parts", "src_part_ids");
      const int64_t arity = arity_parts[i];
      const int64_t pos = pos_parts[i];
      TORCH_CHECK(arity > 0, op, " requires arity > 0 for edge part ", i, ".");
      TORCH_CHECK(pos >= 0 && pos < arity, op, " pos out of range for edge part ", i, ": pos=", pos, " arity=", arity,
                  ".");
      srcs.push_back(edge_src_parts[i]);
      src_mul.push_back(1);
      src_add.push_back(offsets[part]);
      dsts.push_back(edge_dst_parts[i]);
      dst_mul.push_back(arity);
      dst_add.push_back(slot_offset_parts[i] + pos);
   }
   return {x_cat, pack_index(srcs, src_mul, src_add, xs[0]), pack_index(dsts, dst_mul, dst_add, xs[0])};
}

// fanin_pack_from_edges (mp_ops.cpp:2616-2773): edge part k reads message
// rows (src_k * arity_k + pos_k) (mode 0, relation slots) or src_k (mode 1,
// labels) of value part p_k, offset by the rows before it, into dst_k.
std::tuple< Tensor, Tensor, Tensor > fanin_pack_from_edges(at::TensorList rel_parts, at::TensorList edge_src_parts,
                                                           at::TensorList edge_dst_parts, at::IntArrayRef rel_part_ids,
                                                           at::IntArrayRef arity_parts, at::IntArrayRef pos_parts,
                                                           int64_t mode)
{
   const char* op = "fanin_pack_from_edges";
   TORCH_CHECK(!rel_parts.empty(), op, " requires at least one relation tensor.");
   TORCH_CHECK(mode == 0 || mode == 1, op, " mode must be 0 (relation) or 1 (label), got ", mode, ".");
   const size_t n = edge_src_parts.size();
   TORCH_CHECK(edge_dst_parts.size() == n, op, " expects edge_src_parts and edge_dst_parts with equal lengths.");
   TORCH_CHECK(rel_part_ids.size() == n && arity_parts.size() == n && pos_parts.size() == n, op,
               " expects metadata arrays to match number of edge parts.");
   const std::vector< Tensor > rels = rel_parts.vec();
   check_value_parts(rels, op, "rel_parts");
   std::vector< int64_t > offsets;
   int64_t offset = 0;
   for(const auto& r : rels) {
      offsets.push_back(offset);
      offset += r.size(0);
   }
   const Tensor rel_cat = cat_or_single(rels);
   if(n == 0) return {rel_cat, empty_index_like(rels[0]), empty_index_like(rels[0])};
   std::vector< Tensor > srcs, dsts;
   std::vector< int64_t > src_mul, src_add;
   for(size_t i = 0; i < n; ++i) {
      const int64_t part = check_edge_part(edge_src_parts[i], edge_dst_parts[i], rels[0], i, rel_part_ids[i],
                                           rels.size(), op, "rel_parts", "rel_part_ids");
      int64_t mul = 1, add = offsets[part];
      if(mode == 0) {
         const int64_t arity = arity_parts[i];
         const int64_t pos = pos_parts[i];
         TORCH_CHECK(arity > 0, op, " requires arity > 0 in relation mode for edge part ", i, ".");
         TORCH_CHECK(pos >= 0 && pos < arity, op, " pos out of range for edge part ", i, ": pos=", pos,
                     " arity=", arity, ".");
         mul = arity;
         add += pos;
      }
      srcs.push_back(edge_src_parts[i]);
      src_mul.push_back(mul);
      src_add.push_back(add);
      dsts.push_back(edge_dst_parts[i]);
   }
   const std::vector< int64_t > ones(n, 1), zeros(n, 0);
   return {rel_cat, pack_index(srcs, src_mul, src_add, rels[0]), pack_index(dsts, ones, zeros, rels[0])};
}

// build_torch / build_cuda_tag describe the torch this layer was compiled
// against (what the reference loader checks, mp_runtime.py:175-228); the
// kernel library's own metadata follows.

// ---- LGAN ops, sum / mean modes (mp_ops.cpp:3350-3743) ------------------------
//
// Each indexed reduction (mp_common.py:88-118) is a planned sum with its fused
// epilogue: out = base + sum / max(count, 1) (mean) or / max(arity, 1) (pool).
// Plans come from the cache, so the layers of one LGAN forward and backward
// sort each index pair once. int32 indices are accepted as the reference does
// and widened to int64 (a new tensor per call, so their plans are not reused).

constexpr int64_t kModeMean = 2;

void check_int32_or_int64_index(const Tensor& t, const char* name)
{
   check_rank(t, 1, name);
   TORCH_CHECK(t.scalar_type() == at::kLong || t.scalar_type() == at::kInt, name,
               " must have dtype torch.int64 or torch.int32.");
}

Tensor index64(const Tensor& t) { return t.scalar_type() == at::kLong ? contig(t) : t.to(at::kLong).contiguous(); }

// [0, n) on the tensor's device: the gather index of the slot pooling. One
// cached arange per device, grown when needed, so pooling plans stay cached.
Tensor identity_index(int64_t n, const Tensor& like)
{
   static std::mutex mu;
   static std::vector< Tensor > per_device;
   std::lock_guard< std::mutex > lock(mu);
   const int dev = like.device().index();
   if((int)per_device.size() <= dev) per_device.resize(dev + 1);
   Tensor& a = per_device[dev];
   if(!a.defined() || a.numel() < n)
      a = at::arange(std::max< int64_t >(n, 1024), like.options().dtype(at::kLong));
   return a.narrow(0, 0, n);
}

struct LganIndices {
   Tensor rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent;
};

LganIndices lgan_indices(const Tensor& rr_src, const Tensor& rr_dst, const Tensor& tn_rel, const Tensor& tn_ent,
                         const Tensor& nn_rel, const Tensor& nn_ent)
{
   check_int32_or_int64_index(rr_src, "rr_src");
   check_int32_or_int64_index(rr_dst, "rr_dst");
   check_int32_or_int64_index(tn_rel, "tn_rel");
   check_int32_or_int64_index(tn_ent, "tn_ent");
   check_int32_or_int64_index(nn_rel, "nn_rel");
   check_int32_or_int64_index(nn_ent, "nn_ent");
   TORCH_CHECK(rr_src.size(0) == rr_dst.size(0), "rr_src and rr_dst must have equal length.");
   TORCH_CHECK(tn_rel.size(0) == tn_ent.size(0), "tn_rel and tn_ent must have equal length.");
   TORCH_CHECK(nn_rel.size(0) == nn_ent.size(0), "nn_rel and nn_ent must have equal length.");
   return {index64(rr_src), index64(rr_dst), index64(tn_rel), index64(tn_ent), index64(nn_rel), index64(nn_ent)};
}

void check_lgan_mode(int64_t mode, const char* op)
{
   TORCH_CHECK(mode == kModeSum || mode == kModeMean, op, " supports only mode 0=sum or 2=mean.");
}

void check_all_on(const Tensor& ref, std::initializer_list< const Tensor* > ts, const char* op)
{
   for(const Tensor* t : ts)
      TORCH_CHECK(t->device() == ref.device(), op, " expects all tensors on the same device.");
}

// Planned sum with epilogue: out = base + sum / divisor over the plan of (out_index, gather_index).
void planned_sum_ex(const PlanPtr& e, relm_mp_dtype dt, const Tensor& table, const Tensor* base,
                    const int64_t* row_div, bool by_count, Tensor& out, const char* op)
{
   const int64_t emb = table.size(1);
   Tensor scratch = byte_buffer(relm_mp_plan_reduce_scratch_bytes(&e->plan, emb, dt, RELM_MP_MODE_SUM), table);
   check_status(relm_mp_plan_reduce_ex(&e->plan, dt, table.data_ptr(), emb, base ? base->data_ptr() : nullptr,
                                       row_div, by_count ? 1 : 0, out.data_ptr(), scratch.data_ptr(),
                                       (size_t)scratch.numel(), stream_of(table)),
                op);
}

// out[t] = base[t] + (sum of table[src[e]] over dst[e] = t) (/ max(count, 1) in mean mode).
void lgan_forward_agg(relm_mp_dtype dt, const Tensor& table, const Tensor& src, const Tensor& dst, int64_t rows,
                      const char* src_name, const char* dst_name, const Tensor* base, bool mean, Tensor& out,
                      const char* op)
{
   if(src.numel() == 0 || rows == 0 || table.size(1) == 0) {  // mp_ops.cpp:3433-3437
      if(base)
         out.copy_(*base);
      else
         out.zero_();
      return;
   }
   const PlanPtr e = PlanCache::get().lookup(dst, src, rows, rows, table.size(0), dst_name, src_name, false);
   planned_sum_ex(e, dt, table, base, nullptr, mean, out, op);
}

// The reverse (mp_ops.cpp:3527-3555): out[s] = base[s] + sum over src[e] = s of
// grad[dst[e]] (/ max(count of dst[e], 1) in mean mode).
void lgan_reverse_agg(relm_mp_dtype dt, const Tensor& grad, const Tensor& src, const Tensor& dst, int64_t rows,
                      const char* src_name, const char* dst_name, const Tensor* base, bool mean, Tensor& out,
                      const char* op)
{
   if(src.numel() == 0 || rows == 0 || grad.size(1) == 0) {
      if(base)
         out.copy_(*base);
      else
         out.zero_();
      return;
   }
   const PlanPtr e = PlanCache::get().lookup(src, dst, rows, rows, grad.size(0), src_name, dst_name, false);
   Tensor table = grad;
   if(mean) {
      table = at::empty_like(grad);
      const int32_t* counts = PlanCache::get().gather_counts(e, grad);
      check_status(relm_mp_divide_rows(dt, grad.data_ptr(), grad.size(0), grad.size(1), counts, table.data_ptr(),
                                       stream_of(grad)),
                   op);
   }
   planned_sum_ex(e, dt, table, base, nullptr, false, out, op);
}

// The plans of a graph step's forward aggregations (after `first`, the slot
// pooling's, when given), built with one host wait; the conditions are
// lgan_forward_agg's, so exactly the plans it would build are built, in its order.
void lgan_prebuild_forward(const LganIndices& ix, int64_t R, int64_t N, int64_t emb,
                           const PlanCache::Request* first = nullptr)
{
   std::vector< PlanCache::Request > reqs;
   if(first) reqs.push_back(*first);
   if(emb > 0) {
      if(ix.rr_src.numel() > 0 && R > 0) reqs.push_back({&ix.rr_dst, &ix.rr_src, R, R, R, "rr_dst", "rr_src", false});
      if(ix.tn_rel.numel() > 0 && N > 0) reqs.push_back({&ix.tn_ent, &ix.tn_rel, N, N, R, "tn_ent", "tn_rel", false});
      if(ix.nn_rel.numel() > 0 && N > 0) reqs.push_back({&ix.nn_ent, &ix.nn_rel, N, N, R, "nn_ent", "nn_rel", false});
   }
   PlanCache::get().prebuild(reqs);
}

// The same for the backward's reverse aggregations (lgan_reverse_agg's
// conditions and order), then `last`, the slot gradient's pooling plan.
void lgan_prebuild_backward(const LganIndices& ix, int64_t R, int64_t n_tn, int64_t n_nn, int64_t emb,
                            const PlanCache::Request* last = nullptr)
{
   std::vector< PlanCache::Request > reqs;
   if(emb > 0 && R > 0) {
      if(ix.tn_rel.numel() > 0) reqs.push_back({&ix.tn_rel, &ix.tn_ent, R, R, n_tn, "tn_rel", "tn_ent", false});
      if(ix.nn_rel.numel() > 0) reqs.push_back({&ix.nn_rel, &ix.nn_ent, R, R, n_nn, "nn_rel", "nn_ent", false});
      if(ix.rr_src.numel() > 0) reqs.push_back({&ix.rr_src, &ix.rr_dst, R, R, R, "rr_src", "rr_dst", false});
   }
   if(last) reqs.push_back(*last);
   PlanCache::get().prebuild(reqs);
}

// x1 = x + agg_rr(x); tn = agg_tn(x1); nn = agg_nn(x1)
std::tuple< Tensor, Tensor, Tensor > lgan_graph_forward(relm_mp_dtype dt, const Tensor& x, const LganIndices& ix,
                                                        int64_t entity_dim_size, bool mean, const char* op)
{
   const int64_t R = x.size(0), emb = x.size(1);
   lgan_prebuild_forward(ix, R, entity_dim_size, emb);
   Tensor x1 = at::empty({R, emb}, x.options());
   Tensor tn = at::empty({entity_dim_size, emb}, x.options());
   Tensor nn = at::empty({entity_dim_size, emb}, x.options());
   lgan_forward_agg(dt, x, ix.rr_src, ix.rr_dst, R, "rr_src", "rr_dst", &x, mean, x1, op);
   lgan_forward_agg(dt, x1, ix.tn_rel, ix.tn_ent, entity_dim_size, "tn_rel", "tn_ent", nullptr, mean, tn, op);
   lgan_forward_agg(dt, x1, ix.nn_rel, ix.nn_ent, entity_dim_size, "nn_rel", "nn_ent", nullptr, mean, nn, op);
   return {x1, tn, nn};
}

// Gradient of the graph step's input from the gradients of (x1, tn, nn).
Tensor lgan_graph_backward(relm_mp_dtype dt, const Tensor& gx, const Tensor& gtn, const Tensor& gnn,
                           const LganIndices& ix, int64_t relation_count, bool mean, const char* op)
{
   const int64_t emb = gx.size(1);
   lgan_prebuild_backward(ix, relation_count, gtn.size(0), gnn.size(0), emb);
   Tensor g1 = at::empty({relation_count, emb}, gx.options());
   lgan_reverse_agg(dt, gtn, ix.tn_rel, ix.tn_ent, relation_count, "tn_rel", "tn_ent", &gx, mean, g1, op);
   lgan_reverse_agg(dt, gnn, ix.nn_rel, ix.nn_ent, relation_count, "nn_rel", "nn_ent", &g1, mean, g1, op);
   Tensor g0 = at::empty({relation_count, emb}, gx.options());
   lgan_reverse_agg(dt, g1, ix.rr_src, ix.rr_dst, relation_count, "rr_src", "rr_dst", &g1, mean, g0, op);
   return g0;
}

void check_lgan_grads(const Tensor& gx, const Tensor& gtn, const Tensor& gnn, int64_t relation_count, const char* op)
{
   check_rank(gx, 2, "grad_relation_pair_x");
   check_rank(gtn, 2, "grad_tn_msgs");
   check_rank(gnn, 2, "grad_nn_msgs");
   TORCH_CHECK(relation_count >= 0, "relation_count must be >= 0.");
   TORCH_CHECK(gx.size(0) == relation_count, op, ": grad_relation_pair_x must have relation_count rows.");
   TORCH_CHECK(gtn.size(1) == gx.size(1) && gnn.size(1) == gx.size(1) && gtn.size(0) == gnn.size(0), op,
               ": grad_tn_msgs and grad_nn_msgs must be [entity_dim_size, emb] like each other.");
   TORCH_CHECK(gtn.scalar_type() == gx.scalar_type() && gnn.scalar_type() == gx.scalar_type(), op,
               ": the three gradients must share dtype.");
}

// mp_ops.cpp:3574-3656
std::tuple< Tensor, Tensor, Tensor > lgan_relation_graph_step_cuda(const Tensor& relation_pair_x, const Tensor& rr_src,
                                                                   const Tensor& rr_dst, const Tensor& tn_rel,
                                                                   const Tensor& tn_ent, const Tensor& nn_rel,
                                                                   const Tensor& nn_ent, int64_t entity_dim_size,
                                                                   int64_t mode)
{
   const char* op = "lgan_relation_graph_step";
   check_rank(relation_pair_x, 2, "relation_pair_x");
   check_all_on(relation_pair_x, {&rr_src, &rr_dst, &tn_rel, &tn_ent, &nn_rel, &nn_ent},
                "lgan_relation_graph_step");
   TORCH_CHECK(entity_dim_size >= 0, "entity_dim_size must be >= 0.");
   const LganIndices ix = lgan_indices(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent);
   check_lgan_mode(mode, op);
   c10::cuda::CUDAGuard guard(relation_pair_x.device());
   const relm_mp_dtype dt = to_dtype(relation_pair_x, op);
   return lgan_graph_forward(dt, contig(relation_pair_x), ix, entity_dim_size, mode == kModeMean, op);
}

// mp_ops.cpp:3658-3743
Tensor lgan_relation_graph_step_backward_cuda(const Tensor& grad_relation_pair_x, const Tensor& grad_tn_msgs,
                                              const Tensor& grad_nn_msgs, const Tensor& rr_src, const Tensor& rr_dst,
                                              const Tensor& tn_rel, const Tensor& tn_ent, const Tensor& nn_rel,
                                              const Tensor& nn_ent, int64_t relation_count, int64_t mode)
{
   const char* op = "lgan_relation_graph_step_backward";
   check_all_on(grad_relation_pair_x, {&grad_tn_msgs, &grad_nn_msgs, &rr_src, &rr_dst, &tn_rel, &tn_ent, &nn_rel,
                                       &nn_ent},
                op);
   const LganIndices ix = lgan_indices(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent);
   check_lgan_grads(grad_relation_pair_x, grad_tn_msgs, grad_nn_msgs, relation_count, op);
   check_lgan_mode(mode, op);
   c10::cuda::CUDAGuard guard(grad_relation_pair_x.device());
   const relm_mp_dtype dt = to_dtype(grad_relation_pair_x, op);
   return lgan_graph_backward(dt, contig(grad_relation_pair_x), contig(grad_tn_msgs), contig(grad_nn_msgs), ix,
                              relation_count, mode == kModeMean, op);
}

// The slot-pooling plan: output rows = relation instances, gather = slot ids.
PlanPtr pool_plan(const Tensor& slot_to_rel, int64_t relation_count, const Tensor& like)
{
   const int64_t S = slot_to_rel.numel();
   return PlanCache::get().lookup(slot_to_rel, identity_index(S, like), relation_count, relation_count, S,
                                  "slot_to_relation_instance", "slot", false);
}

// mp_ops.cpp:3350-3469
std::tuple< Tensor, Tensor, Tensor > lgan_pool_reduce_cuda(const Tensor& slot_messages,
                                                           const Tensor& slot_to_relation_instance,
                                                           const Tensor& relation_instance_arities,
                                                           const Tensor& rr_src, const Tensor& rr_dst,
                                                           const Tensor& tn_rel, const Tensor& tn_ent,
                                                           const Tensor& nn_rel, const Tensor& nn_ent,
                                                           int64_t entity_dim_size, int64_t mode)
{
   const char* op = "lgan_pool_reduce";
   check_rank(slot_messages, 2, "slot_messages");
   check_int32_or_int64_index(slot_to_relation_instance, "slot_to_relation_instance");
   check_int64_index(relation_instance_arities, "relation_instance_arities");
   check_all_on(slot_messages, {&slot_to_relation_instance, &relation_instance_arities, &rr_src, &rr_dst, &tn_rel,
                                &tn_ent, &nn_rel, &nn_ent},
                op);
   TORCH_CHECK(entity_dim_size >= 0, "entity_dim_size must be >= 0.");
   TORCH_CHECK(slot_to_relation_instance.size(0) == slot_messages.size(0),
               "slot_to_relation_instance length must match slot_messages rows.");
   const LganIndices ix = lgan_indices(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent);
   check_lgan_mode(mode, op);
   c10::cuda::CUDAGuard guard(slot_messages.device());
   const relm_mp_dtype dt = to_dtype(slot_messages, op);
   const Tensor slots = contig(slot_messages);
   const Tensor s2r = index64(slot_to_relation_instance);
   const Tensor arities = contig(relation_instance_arities);
   const int64_t R = arities.size(0), emb = slots.size(1);
   // x[r] = (sum of the slot rows of r) / max(arity[r], 1)  (mp_ops.cpp:3424-3432)
   Tensor x0 = at::empty({R, emb}, slots.options());
   {
      const Tensor ident = identity_index(s2r.numel(), slots);
      const PlanCache::Request pool{&s2r, &ident, R, R, s2r.numel(), "slot_to_relation_instance", "slot", false};
      const bool pooled = !(slots.size(0) == 0 || R == 0 || emb == 0);
      lgan_prebuild_forward(ix, R, entity_dim_size, emb, pooled ? &pool : nullptr);
   }
   if(slots.size(0) == 0 || R == 0 || emb == 0) {
      x0.zero_();
   } else {
      const PlanPtr e = pool_plan(s2r, R, slots);
      planned_sum_ex(e, dt, slots, nullptr, arities.data_ptr< int64_t >(), false, x0, op);
   }
   return lgan_graph_forward(dt, x0, ix, entity_dim_size, mode == kModeMean, op);
}

// mp_ops.cpp:3471-3572
Tensor lgan_pool_reduce_backward_cuda(const Tensor& grad_relation_pair_x, const Tensor& grad_tn_msgs,
                                      const Tensor& grad_nn_msgs, const Tensor& slot_to_relation_instance,
                                      const Tensor& relation_instance_arities, const Tensor& rr_src,
                                      const Tensor& rr_dst, const Tensor& tn_rel, const Tensor& tn_ent,
                                      const Tensor& nn_rel, const Tensor& nn_ent, int64_t relation_count,
                                      int64_t mode)
{
   const char* op = "lgan_pool_reduce_backward";
   check_int32_or_int64_index(slot_to_relation_instance, "slot_to_relation_instance");
   check_int64_index(relation_instance_arities, "relation_instance_arities");
   check_all_on(grad_relation_pair_x, {&grad_tn_msgs, &grad_nn_msgs, &slot_to_relation_instance,
                                       &relation_instance_arities, &rr_src, &rr_dst, &tn_rel, &tn_ent, &nn_rel,
                                       &nn_ent},
                op);
   const LganIndices ix = lgan_indices(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent);
   check_lgan_grads(grad_relation_pair_x, grad_tn_msgs, grad_nn_msgs, relation_count, op);
   check_lgan_mode(mode, op);
   TORCH_CHECK(relation_instance_arities.size(0) >= relation_count,
               "relation_instance_arities must have at least relation_count entries.");
   c10::cuda::CUDAGuard guard(grad_relation_pair_x.device());
   const relm_mp_dtype dt = to_dtype(grad_relation_pair_x, op);
   const Tensor gx = contig(grad_relation_pair_x);
   const Tensor s2r = index64(slot_to_relation_instance);
   {
      const Tensor ident = identity_index(s2r.numel(), gx);
      const PlanCache::Request pool{&s2r, &ident, relation_count, relation_count, s2r.numel(),
                                    "slot_to_relation_instance", "slot", false};
      const bool pooled = s2r.numel() > 0 && gx.size(1) > 0;
      lgan_prebuild_backward(ix, relation_count, grad_tn_msgs.size(0), grad_nn_msgs.size(0), gx.size(1),
                             pooled ? &pool : nullptr);
   }
   const Tensor g0 = lgan_graph_backward(dt, gx, contig(grad_tn_msgs), contig(grad_nn_msgs), ix, relation_count,
                                         mode == kModeMean, op);
   const Tensor arities = contig(relation_instance_arities);
   const int64_t S = s2r.size(0), emb = gx.size(1);
   Tensor grad_slots = at::empty({S, emb}, gx.options());
   if(S == 0 || emb == 0) return grad_slots;
   // grad_slot[s] = g0[r] / max(arity[r], 1) for the relation r of slot s (s2r validated by the pooling plan)
   const PlanPtr e = pool_plan(s2r, relation_count, gx);
   check_status(relm_mp_plan_gather_rows_div(&e->plan, s2r.data_ptr< int64_t >(), dt, g0.data_ptr(), emb,
                                             arities.data_ptr< int64_t >(), grad_slots.data_ptr(), stream_of(gx)),
                op);
   return grad_slots;
}

std::tuple< Tensor, Tensor, Tensor > lgan_pool_reduce_meta(const Tensor& slot_messages, const Tensor&,
                                                           const Tensor& arities, const Tensor&, const Tensor&,
                                                           const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                                                           int64_t entity_dim_size, int64_t)
{
   const int64_t emb = slot_messages.size(1);
   return {at::empty({arities.size(0), emb}, slot_messages.options()),
           at::empty({entity_dim_size, emb}, slot_messages.options()),
           at::empty({entity_dim_size, emb}, slot_messages.options())};
}

Tensor lgan_pool_reduce_backward_meta(const Tensor& grad_relation_pair_x, const Tensor&, const Tensor&,
                                      const Tensor& slot_to_relation_instance, const Tensor&, const Tensor&,
                                      const Tensor&, const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                                      int64_t, int64_t)
{
   return at::empty({slot_to_relation_instance.size(0), grad_relation_pair_x.size(1)},
                    grad_relation_pair_x.options());
}

std::tuple< Tensor, Tensor, Tensor > lgan_relation_graph_step_meta(const Tensor& x, const Tensor&, const Tensor&,
                                                                   const Tensor&, const Tensor&, const Tensor&,
                                                                   const Tensor&, int64_t entity_dim_size, int64_t)
{
   return {at::empty_like(x), at::empty({entity_dim_size, x.size(1)}, x.options()),
           at::empty({entity_dim_size, x.size(1)}, x.options())};
}

Tensor lgan_relation_graph_step_backward_meta(const Tensor& grad_relation_pair_x, const Tensor&, const Tensor&,
                                              const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                                              const Tensor&, const Tensor&, int64_t relation_count, int64_t)
{
   return at::empty({relation_count, grad_relation_pair_x.size(1)}, grad_relation_pair_x.options());
}

std::string build_info()
{
   return std::string("build_torch=") + RELM_MP_BUILD_TORCH_VERSION + ";build_cuda_tag=" + RELM_MP_BUILD_CUDA_TAG
          + ";abi_target=" + RELM_MP_ABI_TARGET + ";abi_lane=nonstable;" + relm_mp_build_info();
}

void clear_plan_cache() { PlanCache::get().clear(); }
std::vector< int64_t > plan_cache_stats() { return PlanCache::get().stats(); }
void set_plan_cache_capacity(int64_t cap) { PlanCache::get().set_capacity(cap); }

}  // namespace relm_b200

TORCH_LIBRARY(relm_mp, m)
{
   m.def(
      "fanout_pack_multi(Tensor[] x_parts, Tensor[] src_idx_parts, Tensor[] flat_dst_parts) -> (Tensor, Tensor, Tensor)"
   );
   m.def(
      "fanout_pack_from_edges(Tensor[] x_parts, Tensor[] edge_src_parts, Tensor[] edge_dst_parts, int[] src_part_ids, "
      "int[] arity_parts, int[] pos_parts, int[] slot_offset_parts) -> (Tensor, Tensor, Tensor)"
   );
   m.def("fanout_scatter(Tensor x_cat, Tensor src_global_idx, Tensor flat_dst, int out_rows) -> Tensor");
   m.def("fanout_scatter_backward(Tensor grad_out, Tensor src_global_idx, Tensor flat_dst, int x_rows) -> Tensor");
   m.def("fanin_reduce(Tensor rel_flat, Tensor flat_src, Tensor dst_idx, int dim_size, int mode) -> Tensor");
   m.def("fanin_reduce_sum_backward(Tensor grad_out, Tensor flat_src, Tensor dst_idx, int rel_rows) -> Tensor");
   m.def(
      "fanin_reduce_logsumexp_backward(Tensor grad_out, Tensor rel_flat, Tensor flat_src, Tensor dst_idx, Tensor out, "
      "int rel_rows) -> Tensor"
   );
   m.def(
      "fanin_pack_multi(Tensor[] rel_parts, Tensor[] flat_src_parts, Tensor[] dst_idx_parts) -> (Tensor, Tensor, Tensor)"
   );
   m.def(
      "fanin_pack_from_edges(Tensor[] rel_parts, Tensor[] edge_src_parts, Tensor[] edge_dst_parts, int[] rel_part_ids, "
      "int[] arity_parts, int[] pos_parts, int mode) -> (Tensor, Tensor, Tensor)"
   );
   m.def(
      "lgan_pool_reduce(Tensor slot_messages, Tensor slot_to_relation_instance, Tensor relation_instance_arities, "
      "Tensor rr_src, Tensor rr_dst, Tensor tn_rel, Tensor tn_ent, Tensor nn_rel, Tensor nn_ent, int entity_dim_size, "
      "int mode) -> (Tensor, Tensor, Tensor)"
   );
   m.def(
      "lgan_pool_reduce_backward(Tensor grad_relation_pair_x, Tensor grad_tn_msgs, Tensor grad_nn_msgs, "
      "Tensor slot_to_relation_instance, Tensor relation_instance_arities, Tensor rr_src, Tensor rr_dst, "
      "Tensor tn_rel, Tensor tn_ent, Tensor nn_rel, Tensor nn_ent, int relation_count, int mode) -> Tensor"
   );
   m.def(
      "lgan_relation_graph_step(Tensor relation_pair_x, Tensor rr_src, Tensor rr_dst, Tensor tn_rel, Tensor tn_ent, "
      "Tensor nn_rel, Tensor nn_ent, int entity_dim_size, int mode) -> (Tensor, Tensor, Tensor)"
   );
   m.def(
      "lgan_relation_graph_step_backward(Tensor grad_relation_pair_x, Tensor grad_tn_msgs, Tensor grad_nn_msgs, "
      "Tensor rr_src, Tensor rr_dst, Tensor tn_rel, Tensor tn_ent, Tensor nn_rel, Tensor nn_ent, int relation_count, "
      "int mode) -> Tensor"
   );
   m.def("build_info() -> str");
}

TORCH_LIBRARY_IMPL(relm_mp, CUDA, m)
{
   m.impl("fanout_scatter", relm_b200::fanout_scatter_cuda);
   m.impl("fanout_scatter_backward", relm_b200::fanout_scatter_backward_cuda);
   m.impl("fanin_reduce", relm_b200::fanin_reduce_cuda);
   m.impl("fanin_reduce_sum_backward", relm_b200::fanin_reduce_sum_backward_cuda);
   m.impl("fanin_reduce_logsumexp_backward", relm_b200::fanin_reduce_logsumexp_backward_cuda);
   m.impl("lgan_pool_reduce", relm_b200::lgan_pool_reduce_cuda);
   m.impl("lgan_pool_reduce_backward", relm_b200::lgan_pool_reduce_backward_cuda);
   m.impl("lgan_relation_graph_step", relm_b200::lgan_relation_graph_step_cuda);
   m.impl("lgan_relation_graph_step_backward", relm_b200::lgan_relation_graph_step_backward_cuda);
}

TORCH_LIBRARY_IMPL(relm_mp, Meta, m)
{
   m.impl("fanout_scatter", relm_b200::fanout_scatter_meta);
   m.impl("fanout_scatter_backward", relm_b200::fanout_scatter_backward_meta);
   m.impl("fanin_reduce", relm_b200::fanin_reduce_meta);
   m.impl("fanin_reduce_sum_backward", relm_b200::fanin_reduce_sum_backward_meta);
   m.impl("fanin_reduce_logsumexp_backward", relm_b200::fanin_reduce_logsumexp_backward_meta);
   m.impl("lgan_pool_reduce", relm_b200::lgan_pool_reduce_meta);
   m.impl("lgan_pool_reduce_backward", relm_b200::lgan_pool_reduce_backward_meta);
   m.impl("lgan_relation_graph_step", relm_b200::lgan_relation_graph_step_meta);
   m.impl("lgan_relation_graph_step_backward", relm_b200::lgan_relation_graph_step_backward_meta);
}

TORCH_LIBRARY_IMPL(relm_mp, CompositeImplicitAutograd, m)
{
   m.impl("fanout_pack_multi", relm_b200::fanout_pack_multi);
   m.impl("fanout_pack_from_edges", relm_b200::fanout_pack_from_edges);
   m.impl("fanin_pack_multi", relm_b200::fanin_pack_multi);
   m.impl("fanin_pack_from_edges", relm_b200::fanin_pack_from_edges);
   m.impl("build_info", relm_b200::build_info);
}

// Ops of this package outside the reference namespace: plan-cache control and
// the smoothed logsumexp of relmo's models.
TORCH_LIBRARY(relm_mp_b200, m)
{
   m.def("clear_plan_cache() -> ()", relm_b200::clear_plan_cache);
   m.def("plan_cache_stats() -> int[]", relm_b200::plan_cache_stats);
   m.def("set_plan_cache_capacity(int capacity) -> ()", relm_b200::set_plan_cache_capacity);
   m.def(
      "fanin_reduce_smoothed_logsumexp(Tensor rel_flat, Tensor flat_src, Tensor dst_idx, int dim_size, float beta, "
      "float eps) -> Tensor"
   );
   m.def(
      "fanin_reduce_smoothed_logsumexp_backward(Tensor grad_out, Tensor rel_flat, Tensor flat_src, Tensor dst_idx, "
      "Tensor out, int rel_rows, float beta) -> Tensor"
   );
}

TORCH_LIBRARY_IMPL(relm_mp_b200, CUDA, m)
{
   m.impl("fanin_reduce_smoothed_logsumexp", relm_b200::smoothed_logsumexp_cuda);
   m.impl("fanin_reduce_smoothed_logsumexp_backward", relm_b200::smoothed_logsumexp_backward_cuda);
}

TORCH_LIBRARY_IMPL(relm_mp_b200, Meta, m)
{
   m.impl("fanin_reduce_smoothed_logsumexp", relm_b200::smoothed_logsumexp_meta);
   m.impl("fanin_reduce_smoothed_logsumexp_backward", relm_b200::smoothed_logsumexp_backward_meta);
}
