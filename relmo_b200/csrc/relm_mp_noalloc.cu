// fanin_reduce without any device allocation, for callers that cannot
// allocate device memory at the point of the call.
//
// Some hosts of this library must not call cudaMalloc (or any allocating
// routine) where they run the op: their device memory belongs to another
// allocator they cannot reach from there, or they cannot afford the implicit
// device synchronization cudaMalloc brings while other work is in flight. This
// entry point takes its whole workspace (plan and reduction scratch) from one
// file-scope static device array, so a call allocates nothing; the caller
// still passes the inputs and the output.
//
// This file holds no kernel, so its module is loaded on the first call on a
// device (CUDA loads modules lazily by default): that call commits the
// RELM_MP_NOALLOC_SCRATCH_BYTES array on the device, and the load may
// synchronize the device. From then on the device holds the array until the
// process exits. Callers make one warm-up call per device at set-up (or run
// with CUDA_MODULE_LOADING=EAGER, which loads it with the library). All calls
// on a device share the array: calls whose work overlaps on the GPU (different
// streams, different host threads) race on it.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>

#include "relm_mp_internal.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[RELM_MP_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::atomic< void* > g_scratch_ptr[kMaxDevices];

// Device address of the static scratch on the current device. Host code sees
// g_noalloc_scratch only as a host-side stand-in symbol, so the address comes
// from cudaGetSymbolAddress, looked up once per device with that device
// current and kept for the later calls (no lock: two threads racing on the
// first call store the same address). A cudaDeviceReset after the first call
// is not supported: the module may reload elsewhere and the kept address
// would be stale.
int scratch_address(void** out)
{
   int dev = -1;
   int rc = relm_mp::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
   if(rc) return rc;
   if(dev < 0 || dev >= kMaxDevices) return relm_mp::fail(RELM_MP_ERR_UNSUPPORTED, "device index out of range.");
   void* ptr = g_scratch_ptr[dev].load(std::memory_order_acquire);
   if(!ptr) {
      rc = relm_mp::check_cuda(cudaGetSymbolAddress(&ptr, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
      if(rc) return rc;
      g_scratch_ptr[dev].store(ptr, std::memory_order_release);
   }
   *out = ptr;
   return RELM_MP_OK;
}

}  // namespace

extern "C" int relm_mp_fanin_reduce_noalloc(relm_mp_dtype dtype, const void* rel_flat, int64_t rel_rows,
                                            int64_t emb, const int64_t* flat_src, const int64_t* dst_idx,
                                            int64_t num_edges, int64_t dim_size, int mode, void* out,
                                            void* stream)
{
   const size_t need = relm_mp_fanin_reduce_workspace_bytes(num_edges, dim_size, emb, dtype, mode);
   if(need > (size_t)RELM_MP_NOALLOC_SCRATCH_BYTES) {
      char msg[256];
      snprintf(
         msg,
         sizeof msg,
         "fanin_reduce_noalloc: %lld edges into %lld rows of %lld needs %zu bytes of scratch; the static scratch "
         "holds %zu bytes. Use relm_mp_fanin_reduce with a caller workspace.",
         (long long)num_edges,
         (long long)dim_size,
         (long long)emb,
         need,
         (size_t)RELM_MP_NOALLOC_SCRATCH_BYTES
      );
      return relm_mp::fail(RELM_MP_ERR_WORKSPACE_TOO_SMALL, msg);
   }
   void* scratch = nullptr;
   const int rc = scratch_address(&scratch);
   if(rc) return rc;
   // The op writes every word of the workspace it reads (memsets for the
   // counters and flags that start at zero), so the previous call's contents
   // need no clearing here.
   return relm_mp_fanin_reduce(
      dtype, rel_flat, rel_rows, emb, flat_src, dst_idx, num_edges, dim_size, mode, out, scratch,
      (size_t)RELM_MP_NOALLOC_SCRATCH_BYTES, stream
   );
}
