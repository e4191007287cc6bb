// Internal declarations shared by the relm_mp CUDA sources.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "relm_mp.h"

namespace relm_mp {

// Merge-path tiles: one warp owns one tile of `items` (output rows + edges).
// The tile size is chosen from the problem size alone, aiming at about
// kTargetTiles tiles (4 resident waves of 32 warps on each of the B200's 148
// SMs), within [kMinTileItems, kMaxTileItems].
#ifndef RELM_MP_TARGET_TILES
#define RELM_MP_TARGET_TILES (148 * 128)
#endif
constexpr int64_t kTargetTiles = RELM_MP_TARGET_TILES;
constexpr int kMinTileItems = 128;
constexpr int kMaxTileItems = 4096;
int plan_tile_items(int64_t num_edges, int64_t num_rows);
// Tiles with a head partial whose row spans more than this many tiles are
// combined by the block-wide long-row fixup instead of a single warp.
constexpr int kLongRowTiles = 64;
// Plans whose rows all hold at most this many edges are reduced a lane group
// per row (k_seg_rows_packed) when the row size allows it; the plan build sets
// device flag [1] when some row is longer (merge-path kernels then).
constexpr int kShortRowEdges = 32;
constexpr int kThreads = 256;

// Alignment of every sub-buffer carved out of a workspace.
constexpr size_t kAlign = 256;

inline size_t align_up(size_t v, size_t a = kAlign) { return (v + a - 1) / a * a; }

// Thread-local error message; returns `status` for convenient `return fail(...)`.
int fail(int status, const std::string& message);
int check_cuda(cudaError_t err, const char* what);
int check_launch(const char* what);

// Carves consecutive aligned sub-buffers out of one workspace.
struct Carver {
   char* base;
   size_t used = 0;
   explicit Carver(void* p) : base(static_cast<char*>(p)) {}
   template <typename T>
   T* take(size_t count)
   {
      T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
      used += align_up(count * sizeof(T));
      return p;
   }
};

// Builds a plan with a separate validation bound for the output index
// (`out_bound` <= num_rows; rows >= out_bound may exist but receive no edges).
// kBuildStart validates and queues the copy of the statistics into host_stats
// (pinned host memory), kBuildFinish (same arguments, after the caller waited
// for the stream) checks them and lays the plan out; kBuildAll does both with
// its own wait. kBuildTrusted lays out indices the caller has validated
// against the same bounds already: no checks, no statistics copy, no host wait,
// and the output index is sorted without looking at its order first.
enum BuildPhase : int { kBuildAll = 0, kBuildStart = 1, kBuildFinish = 2, kBuildTrusted = 3 };
int plan_build_bounded(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                       int64_t num_rows, int64_t out_bound, int64_t gather_rows,
                       const char* out_name, const char* gather_name, bool gather_checked_first,
                       void* plan_mem, size_t plan_bytes, void* scratch, size_t scratch_bytes,
                       cudaStream_t stream, relm_mp_plan* plan, uint32_t* cover = nullptr,
                       int* gather_repeats = nullptr, int64_t* gather_covered = nullptr,
                       BuildPhase phase = kBuildAll, void* host_stats = nullptr);

int64_t plan_num_tiles(int64_t num_edges, int64_t num_rows);

// Element-wise fill of `count` elements of dtype with 0 or -inf.
int fill_rows(relm_mp_dtype dtype, void* out, int64_t count, bool neg_inf, cudaStream_t stream);
// out[0..count) = value (converted to the storage type).
int fill_value(relm_mp_dtype dtype, void* out, int64_t count, double value, cudaStream_t stream);

size_t dtype_size(relm_mp_dtype dtype);

// Stable LSD radix sort of (key, value) pairs by key bits [0, end_bit)
// (relm_mp_sort.cu). The pairs start in (keys, vals) and end in them, or in
// (keys_alt, vals_alt) when *in_alt is set (odd pass counts).
int radix_sort_passes(int end_bit);
size_t radix_sort_temp_bytes(int64_t n, int end_bit);
int radix_sort_pairs(uint32_t* keys, uint32_t* keys_alt, int32_t* vals, int32_t* vals_alt, int64_t n, int end_bit,
                     void* temp, size_t temp_bytes, cudaStream_t stream, bool* in_alt);
// out = inclusive max-scan of in[0, n) (in == out allowed).
size_t scan_i32_temp_bytes(int64_t n);
int scan_max_inclusive(const int32_t* in, int32_t* out, int64_t n, void* temp, size_t temp_bytes,
                       cudaStream_t stream);

}  // namespace relm_mp
