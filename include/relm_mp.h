/*
 * relm_mp.h - C ABI of the B200 (sm_100a) fan-out / fan-in message-passing
 * library (librelm_mp_b200.so).
 *
 * The entry points replace the five hot ops of relmo's torch library
 * `relm_mp` (maichmueller/relmo, src/_ops/mp/mp_ops.cpp). Each `relm_mp_<op>`
 * function computes what `torch.ops.relm_mp.<op>` computes, with plain device
 * pointers, sizes, a caller-provided workspace and a CUDA stream instead of
 * torch tensors:
 *
 *   relm_mp_fanout_scatter            <- fanout_scatter            (mp_ops.cpp:3038-3101, schema 3760-3762)
 *   relm_mp_fanout_scatter_backward   <- fanout_scatter_backward   (mp_ops.cpp:3103-3166, schema 3763-3765)
 *   relm_mp_fanin_reduce              <- fanin_reduce, mode 0 / 1  (mp_ops.cpp:3327-3348, 3168-3222, 3005-3036;
 *                                                                   schema 3766-3768)
 *   relm_mp_fanin_reduce_sum_backward <- fanin_reduce_sum_backward (mp_ops.cpp:3224-3284, schema 3769-3771)
 *   relm_mp_fanin_reduce_logsumexp_backward
 *                                     <- fanin_reduce_logsumexp_backward (mp_ops.cpp:3286-3325, schema 3772-3774)
 *   relm_mp_build_info                <- build_info                (mp_ops.cpp:3745-3749)
 *
 * Conventions shared by every entry point:
 *  - All array pointers are device pointers on the current CUDA device; value
 *    arrays are dense row-major [rows, emb]; index arrays are int64.
 *  - `stream` is a cudaStream_t passed as void*. Work is enqueued on it.
 *  - Outputs are fully written (rows nothing maps to get 0, or -inf for
 *    logsumexp), like the reference's at::zeros / at::full(-inf) outputs.
 *  - `workspace` is device memory of at least the size the matching
 *    `*_workspace_bytes` function returns (256-byte aligned). The library never
 *    allocates device memory itself.
 *  - Index arrays are validated before any output is written. An out-of-range
 *    index returns RELM_MP_ERR_INDEX_OUT_OF_RANGE with a message such as
 *    "flat_dst index out of bounds: 3 not in [0, 3)." (the reference CPU
 *    message, mp_ops.cpp:59-64). Validation reads a few bytes back to the host,
 *    so every call synchronizes `stream` once.
 *  - Return value 0 (RELM_MP_OK) or a relm_mp_status code; relm_mp_last_error()
 *    holds the message of the last failing call on the calling thread.
 *  - Limits: num_edges + rows < 2^31 for every index space.
 *  - Deterministic: the same inputs give bit-identical outputs; there are no
 *    floating-point atomics.
 */
#ifndef RELM_MP_H
#define RELM_MP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RELM_MP_ABI_VERSION 1

#if defined(_WIN32)
#define RELM_MP_API __declspec(dllexport)
#else
#define RELM_MP_API __attribute__((visibility("default")))
#endif

typedef enum relm_mp_dtype {
   RELM_MP_FLOAT32 = 0,
   RELM_MP_FLOAT64 = 1,
   RELM_MP_BFLOAT16 = 2, /* stored bf16, accumulated in fp32 */
   RELM_MP_FLOAT16 = 3   /* stored fp16, accumulated in fp32 */
} relm_mp_dtype;

typedef enum relm_mp_status {
   RELM_MP_OK = 0,
   RELM_MP_ERR_INVALID_ARGUMENT = 1,
   RELM_MP_ERR_INDEX_OUT_OF_RANGE = 2,
   RELM_MP_ERR_WORKSPACE_TOO_SMALL = 3,
   RELM_MP_ERR_UNSUPPORTED = 4,
   RELM_MP_ERR_CUDA = 5
} relm_mp_status;

/* fanin_reduce modes, as relmo.ops.mp_constants MODE_SUM / MODE_LOGSUMEXP. */
#define RELM_MP_MODE_SUM 0
#define RELM_MP_MODE_LOGSUMEXP 1
/* Only for relm_mp_plan_reduce_scratch_bytes: scratch of relm_mp_plan_logsumexp_backward. */
#define RELM_MP_MODE_LOGSUMEXP_BACKWARD 2

/* Static strings: status name; "key=value;..." build metadata. */
RELM_MP_API const char* relm_mp_status_string(int status);
RELM_MP_API const char* relm_mp_build_info(void);
/* Message of the last failing call on the calling thread ("" if none). */
RELM_MP_API const char* relm_mp_last_error(void);
/* Number of kernels this library has launched in the process (every kernel
 * is its own, the plan build's radix sort and scans included). */
RELM_MP_API unsigned long long relm_mp_kernel_launches(void);

/* ---------------------------------------------------------------------------
 * Op-level entry points (one call = one reference op call).
 * ------------------------------------------------------------------------- */

/* fanout_scatter: out[out_rows, emb] = 0; out[flat_dst[e]] = x_cat[src_global_idx[e]].
 * With repeated flat_dst values the highest edge index wins, as the
 * reference CPU loop (mp_ops.cpp:2815-2836) leaves it. When every slot is
 * written at most once (the model's routing) the op runs in source-row order
 * and reads each x row once; otherwise it orders by slot. */
RELM_MP_API size_t relm_mp_fanout_scatter_workspace_bytes(int64_t num_edges, int64_t x_rows, int64_t out_rows,
                                                          int64_t emb, relm_mp_dtype dtype);
RELM_MP_API int relm_mp_fanout_scatter(relm_mp_dtype dtype, const void* x_cat, int64_t x_rows, int64_t emb,
                           const int64_t* src_global_idx, const int64_t* flat_dst,
                           int64_t num_edges, int64_t out_rows, void* out, void* workspace,
                           size_t workspace_bytes, void* stream);

/* fanout_scatter_backward: grad_x[x_rows, emb] = 0;
 * grad_x[src_global_idx[e]] += grad_out[flat_dst[e]]. */
RELM_MP_API size_t relm_mp_fanout_scatter_backward_workspace_bytes(int64_t num_edges, int64_t x_rows,
                                                       int64_t emb, relm_mp_dtype dtype);
RELM_MP_API int relm_mp_fanout_scatter_backward(relm_mp_dtype dtype, const void* grad_out,
                                    int64_t grad_out_rows, int64_t emb,
                                    const int64_t* src_global_idx, const int64_t* flat_dst,
                                    int64_t num_edges, int64_t x_rows, void* grad_x,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* fanin_reduce: mode 0: out[dim_size, emb] = 0; out[dst_idx[e]] += rel_flat[flat_src[e]].
 * mode 1: out[n] = log(sum over edges into n of exp(rel_flat[flat_src[e]])),
 * -inf for rows without edges, computed in one pass with a running
 * (max, sum-exp) pair per column. */
RELM_MP_API size_t relm_mp_fanin_reduce_workspace_bytes(int64_t num_edges, int64_t dim_size, int64_t emb,
                                            relm_mp_dtype dtype, int mode);
RELM_MP_API int relm_mp_fanin_reduce(relm_mp_dtype dtype, const void* rel_flat, int64_t rel_rows, int64_t emb,
                         const int64_t* flat_src, const int64_t* dst_idx, int64_t num_edges,
                         int64_t dim_size, int mode, void* out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* fanin_reduce_sum_backward: grad_rel[rel_rows, emb] = 0;
 * grad_rel[flat_src[e]] += grad_out[dst_idx[e]]. */
RELM_MP_API size_t relm_mp_fanin_reduce_sum_backward_workspace_bytes(int64_t num_edges, int64_t rel_rows,
                                                         int64_t emb, relm_mp_dtype dtype);
RELM_MP_API int relm_mp_fanin_reduce_sum_backward(relm_mp_dtype dtype, const void* grad_out,
                                      int64_t grad_out_rows, int64_t emb, const int64_t* flat_src,
                                      const int64_t* dst_idx, int64_t num_edges, int64_t rel_rows,
                                      void* grad_rel, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* fanin_reduce_logsumexp_backward: grad_rel[rel_rows, emb] = 0;
 * grad_rel[flat_src[e]] += grad_out[dst_idx[e]] * exp(rel_flat[flat_src[e]] - out[dst_idx[e]]).
 * grad_out and out are [dim_size, emb]; rel_flat is [rel_table_rows, emb]. */
RELM_MP_API size_t relm_mp_fanin_reduce_logsumexp_backward_workspace_bytes(int64_t num_edges,
                                                               int64_t rel_rows, int64_t emb,
                                                               relm_mp_dtype dtype);
RELM_MP_API int relm_mp_fanin_reduce_logsumexp_backward(relm_mp_dtype dtype, const void* grad_out,
                                            const void* rel_flat, int64_t rel_table_rows,
                                            const void* out, int64_t dim_size, int64_t emb,
                                            const int64_t* flat_src, const int64_t* dst_idx,
                                            int64_t num_edges, int64_t rel_rows, void* grad_rel,
                                            void* workspace, size_t workspace_bytes,
                                            void* stream);

/* fanin_reduce for callers that cannot allocate device memory where they call
 * it (their device memory belongs to another allocator, or they cannot afford
 * cudaMalloc's implicit device synchronization while other work is in
 * flight). No counterpart in the reference library: it is relm_mp_fanin_reduce
 * with its workspace taken from a static device array of
 * RELM_MP_NOALLOC_SCRATCH_BYTES inside the library. The call allocates
 * nothing. Problems whose workspace (relm_mp_fanin_reduce_workspace_bytes)
 * exceeds that size are rejected with RELM_MP_ERR_WORKSPACE_TOO_SMALL.
 *  - The first call on a device loads the library's module that holds the
 *    array (CUDA loads modules lazily by default), which commits the array on
 *    that device and may synchronize the device, and looks up the array's
 *    device address. Make one warm-up call per device at set-up, before any
 *    stream capture (or run with CUDA_MODULE_LOADING=EAGER). From then on the
 *    device holds the array until exit. A cudaDeviceReset after that first
 *    call is not supported (the kept address would be stale).
 *  - Like relm_mp_fanin_reduce, every call reads its index validation result
 *    back to the host: it blocks the calling thread until `stream` drains.
 *  - All calls on a device share the array: calls that overlap on the GPU
 *    (other streams, other threads) race. */
#define RELM_MP_NOALLOC_SCRATCH_BYTES (16u << 20)
RELM_MP_API int relm_mp_fanin_reduce_noalloc(relm_mp_dtype dtype, const void* rel_flat, int64_t rel_rows,
                                             int64_t emb, const int64_t* flat_src, const int64_t* dst_idx,
                                             int64_t num_edges, int64_t dim_size, int mode, void* out,
                                             void* stream);

/* ---------------------------------------------------------------------------
 * Plans: the CSR of one index pair, reusable across calls.
 *
 * A plan orders the edges by an output index (stable: equal output rows keep
 * edge order) and records, per output row, its edge range and, per edge, the
 * row of the gathered table. Every op above builds one plan and runs one
 * planned kernel; callers that apply the same indices many times (the layers
 * of one RelationalGNN forward and its backward) build the plan once and call
 * the planned entry points. The plan lives in caller memory (`plan_mem`,
 * relm_mp_plan_bytes) and must not be freed while in use; `scratch`
 * (relm_mp_plan_scratch_bytes) is only used during the build.
 * ------------------------------------------------------------------------- */

#define RELM_MP_PLAN_SORTED_INPUT 1u /* out_index was already non-decreasing */
/* Host copies of the plan's device flags (set by relm_mp_plan_read_flags, or
 * by a caller that copied device_flags[0..1] itself): when KNOWN is set, the
 * planned reductions launch only the kernel family the plan needs instead of
 * all of them (the others would return at once on the device). */
#define RELM_MP_PLAN_FLAGS_KNOWN 2u
#define RELM_MP_PLAN_REPEATS 4u   /* device_flags[0]: some row holds more than one edge */
#define RELM_MP_PLAN_LONG_ROWS 8u /* device_flags[1]: some row holds more than 32 edges */
/* Set by a build whose gather index is the identity (gather_index[e] == e for
 * every edge; e.g. the message-row index of a fan-in). */
#define RELM_MP_PLAN_GATHER_IDENTITY 16u

typedef struct relm_mp_plan {
   int64_t num_edges;
   int64_t num_rows;        /* output rows */
   int64_t gather_rows;     /* rows of the gathered table */
   int64_t num_tiles;       /* merge-path tiles over num_rows + num_edges items */
   int32_t tile_items;      /* items per tile */
   uint32_t flags;          /* RELM_MP_PLAN_* */
   const int32_t* row_ptr;  /* device [num_rows + 1]: edges of row r are [row_ptr[r], row_ptr[r+1]) */
   const int32_t* gidx;     /* device [num_edges]: gathered row of the j-th edge in row order */
   const int32_t* tile_row; /* device [num_tiles + 1]: first row of each tile */
   const int32_t* tile_edge;/* device [num_tiles + 1]: first edge of each tile */
   const int32_t* device_flags; /* device [4]: [0] nonzero when some row has more than one
                                   edge, [1] when some row has more than 32; kernels read
                                   them on the device (no host copy needed) */
} relm_mp_plan;

RELM_MP_API size_t relm_mp_plan_bytes(int64_t num_edges, int64_t num_rows);
RELM_MP_API size_t relm_mp_plan_scratch_bytes(int64_t num_edges, int64_t num_rows);
/* Validates out_index in [0, num_rows) and gather_index in [0, gather_rows)
 * (names are used in error messages; NULL gives "out_index"/"gather_index"),
 * then builds the plan. Synchronizes `stream` once. A NULL gather_index is
 * the identity (edge e gathers row e), e.g. the pooling of slot rows. */
RELM_MP_API int relm_mp_plan_build(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                       int64_t num_rows, int64_t gather_rows, const char* out_index_name,
                       const char* gather_index_name, void* plan_mem, size_t plan_bytes,
                       void* scratch, size_t scratch_bytes, void* stream, relm_mp_plan* plan);

/* As relm_mp_plan_build, with a separate validation bound for out_index
 * (out_bound <= num_rows: rows >= out_bound exist but receive no edges) and
 * the order in which the two indices are checked at the same edge
 * (gather_checked_first != 0: gather_index first), which decides the error
 * message when one edge has both out of range. */
RELM_MP_API int relm_mp_plan_build_ex(const int64_t* out_index, const int64_t* gather_index,
                                      int64_t num_edges, int64_t num_rows, int64_t out_bound,
                                      int64_t gather_rows, const char* out_index_name,
                                      const char* gather_index_name, int gather_checked_first,
                                      void* plan_mem, size_t plan_bytes, void* scratch,
                                      size_t scratch_bytes, void* stream, relm_mp_plan* plan);

/* The plan of the identity output index over [0, num_edges) (row r <
 * num_edges holds edge r, rows up to num_rows hold none) and `gather_index`,
 * built without validation and without a host wait: gather_index must
 * already be known to lie in [0, gather_rows), e.g. because the build of
 * another plan over the same index validated it. A fan-in's backward over
 * flat_src = arange uses it with the forward plan's destination index (the
 * forward plan's flags carry RELM_MP_PLAN_GATHER_IDENTITY). The result has
 * RELM_MP_PLAN_FLAGS_KNOWN set. No counterpart in the reference. */
RELM_MP_API int relm_mp_plan_build_identity(const int64_t* gather_index, int64_t num_edges, int64_t num_rows,
                                            int64_t gather_rows, void* plan_mem, size_t plan_bytes, void* stream,
                                            relm_mp_plan* plan);

/* The plan of an (output index, gather index) pair the caller has validated
 * already, against num_rows and gather_rows (e.g. the transposed pair of a
 * plan built before: its gather index is this output index and the other way
 * round, with the same bounds): both are narrowed to int32 and the output
 * index is sorted, with no bounds checks and no host wait. Indices out of
 * range are undefined behaviour here. No counterpart in the reference (its
 * ops keep no plans). */
RELM_MP_API int relm_mp_plan_build_trusted(const int64_t* out_index, const int64_t* gather_index,
                                           int64_t num_edges, int64_t num_rows, int64_t gather_rows,
                                           void* plan_mem, size_t plan_bytes, void* scratch,
                                           size_t scratch_bytes, void* stream, relm_mp_plan* plan);

/* relm_mp_plan_build_ex in two halves, so that the builds of several plans
 * (the three or four index pairs of one LGAN op) share one host wait:
 * relm_mp_plan_build_start validates the indices and queues the copy of the
 * validation's result into `host_stats` (pinned host memory of
 * relm_mp_plan_stats_bytes() bytes); once the caller has waited for `stream`
 * (once for every build it started), relm_mp_plan_build_finish, with the same
 * arguments, memory and scratch, raises the index error if there was one and
 * lays the plan out without another wait. plan_mem, scratch and host_stats
 * must stay untouched between the two calls. No counterpart in the
 * reference (its ops keep no plans). */
RELM_MP_API size_t relm_mp_plan_stats_bytes(void);
RELM_MP_API int relm_mp_plan_build_start(const int64_t* out_index, const int64_t* gather_index,
                                         int64_t num_edges, int64_t num_rows, int64_t out_bound,
                                         int64_t gather_rows, void* plan_mem, size_t plan_bytes,
                                         void* scratch, size_t scratch_bytes, void* host_stats, void* stream);
RELM_MP_API int relm_mp_plan_build_finish(const int64_t* out_index, const int64_t* gather_index,
                                          int64_t num_edges, int64_t num_rows, int64_t out_bound,
                                          int64_t gather_rows, const char* out_index_name,
                                          const char* gather_index_name, int gather_checked_first,
                                          void* plan_mem, size_t plan_bytes, void* scratch,
                                          size_t scratch_bytes, const void* host_stats, void* stream,
                                          relm_mp_plan* plan);

/* relm_mp_plan_build_ex that also computes the coverage of the gather index
 * over [0, gather_rows) in its validation pass: bit g of `cover` (device
 * uint32 [relm_mp_cover_words(gather_rows)], the layout of
 * relm_mp_plan_gather_cover) is set when some edge gathers row g, and
 * *gather_repeats = 1 when some row is gathered more than once,
 * *gather_covered (may be NULL) = the number of distinct gathered rows. No host sync
 * beyond the build's own (the repeat flag comes back with its validation
 * stats). Scratch: relm_mp_plan_cover_scratch_bytes. No counterpart in the
 * reference (its ops keep no plans). */
RELM_MP_API size_t relm_mp_plan_cover_scratch_bytes(int64_t num_edges, int64_t num_rows, int64_t gather_rows);
RELM_MP_API int relm_mp_plan_build_cover(const int64_t* out_index, const int64_t* gather_index, int64_t num_edges,
                                         int64_t num_rows, int64_t out_bound, int64_t gather_rows,
                                         const char* out_index_name, const char* gather_index_name,
                                         int gather_checked_first, void* plan_mem, size_t plan_bytes, void* scratch,
                                         size_t scratch_bytes, uint32_t* cover, int* gather_repeats,
                                         int64_t* gather_covered, void* stream, relm_mp_plan* plan);

/* Copies device_flags[0..1] into plan->flags (RELM_MP_PLAN_FLAGS_KNOWN,
 * RELM_MP_PLAN_REPEATS, RELM_MP_PLAN_LONG_ROWS). Synchronizes `stream`. */
RELM_MP_API int relm_mp_plan_read_flags(relm_mp_plan* plan, void* stream);

/* Scratch for the planned reductions (partials of rows that span tiles). */
RELM_MP_API size_t relm_mp_plan_reduce_scratch_bytes(const relm_mp_plan* plan, int64_t emb,
                                         relm_mp_dtype dtype, int mode);

/* Index packing of the pack ops (fanout_pack_multi, fanin_pack_multi,
 * fanout_pack_from_edges, fanin_pack_from_edges; mp_ops.cpp:412-570,
 * 2511-2773): out[start_k + i] = parts[k].src[i] * parts[k].mul + parts[k].add
 * for every part k in order (start_k = sum of the earlier parts' len), i.e. the
 * per-part offset / arity arithmetic and the concatenation of all parts, in
 * one kernel launch per 64 parts. `parts` is a host array; src and out are
 * device int64 arrays; parts with len 0 are skipped. */
typedef struct relm_mp_index_part {
   const int64_t* src;
   int64_t len;
   int64_t mul;
   int64_t add;
} relm_mp_index_part;
RELM_MP_API int relm_mp_pack_index(const relm_mp_index_part* parts, int num_parts, int64_t* out, void* stream);

/* 32-bit words of a cover bitmap over `rows` rows. */
static inline size_t relm_mp_cover_words(int64_t rows) { return rows > 0 ? (size_t)((rows + 31) / 32) : 1u; }

/* Coverage of the plan's gather index over [0, gather_rows): bit g of the
 * bitmap (word g / 32, bit g % 32; device uint32 [relm_mp_cover_words(gather_rows)])
 * is set when some edge gathers row g; *has_dups = 1 when some row is gathered
 * more than once. Synchronizes `stream` once. */
RELM_MP_API int relm_mp_plan_gather_cover(const relm_mp_plan* plan, uint32_t* cover, int* has_dups,
                                          void* stream);
/* relm_mp_plan_gather_cover with caller scratch
 * (relm_mp_plan_gather_cover_scratch_bytes: one byte per gathered row): the
 * gathered rows are marked with plain byte stores and packed into the bitmap,
 * and repeats are found by counting the distinct rows, instead of one L2
 * atomic per edge. Same results; synchronizes `stream` once. *covered_rows (may
 * be NULL): the number of distinct gathered rows. */
RELM_MP_API size_t relm_mp_plan_gather_cover_scratch_bytes(const relm_mp_plan* plan);
RELM_MP_API int relm_mp_plan_gather_cover_ex(const relm_mp_plan* plan, uint32_t* cover, int* has_dups,
                                             int64_t* covered_rows, void* scratch, size_t scratch_bytes,
                                             void* stream);
/* Number of the plan's output rows that hold at least one edge (counted by
 * the plan build on the device). Synchronizes `stream` once. No counterpart in
 * the reference (its ops keep no plans). */
RELM_MP_API int relm_mp_plan_nonempty_rows(const relm_mp_plan* plan, int64_t* rows, void* stream);
/* Scatter in plan-row order, for a gather index that covers each row at most
 * once: out[gidx[j]] = table[r] for every edge j of plan row r, and 0 in the
 * out rows `cover` marks as uncovered (cover NULL: every out row is gathered by
 * some edge, nothing is zeroed). fanout forward through the source plan
 * (plan rows = x rows, gather index = flat_dst): every x row is read once. */
RELM_MP_API int relm_mp_plan_scatter_rows(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* table,
                                          int64_t emb, const uint32_t* cover, void* out, void* stream);
/* Logsumexp backward (mp_ops.cpp:3286-3325) through the FORWARD's plan (output
 * rows = destination rows, gather index = flat_src), for a flat_src that uses
 * each message row at most once (cover from relm_mp_plan_gather_cover, no
 * repeats): grad_rel[m] = grad_out[d] * exp(rel[m] - lse_out[d]) for every edge
 * (d, m), 0 for message rows no edge uses (cover NULL: every message row is
 * used, nothing is zeroed). Reads each destination row's
 * grad_out / lse_out once instead of once per message; rows of 16..256 bytes
 * (a power of two times 16) with 16-byte aligned tables, else UNSUPPORTED. */
RELM_MP_API int relm_mp_plan_scatter_logsumexp_backward(const relm_mp_plan* plan, relm_mp_dtype dtype,
                                                        const void* grad_out, const void* lse_out,
                                                        const void* rel, int64_t emb, const uint32_t* cover,
                                                        void* grad_rel, void* stream);
/* out[r] = table[gidx[last edge of r]] or 0 for rows without edges (fanout forward). */
RELM_MP_API int relm_mp_plan_gather_last(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* table,
                             int64_t emb, void* out, void* stream);
/* mode 0: out[r] = sum of table[gidx[j]] over the edges j of r;
 * mode 1: out[r] = log(sum of exp(table[gidx[j]])), -inf when r has no edges. */
RELM_MP_API int relm_mp_plan_reduce(const relm_mp_plan* plan, relm_mp_dtype dtype, int mode, const void* table,
                        int64_t emb, void* out, void* scratch, size_t scratch_bytes, void* stream);
/* grad_rel[r] = sum over edges j of r of grad_out[gidx[j]] * exp(rel[r] - lse_out[gidx[j]]). */
RELM_MP_API int relm_mp_plan_logsumexp_backward(const relm_mp_plan* plan, relm_mp_dtype dtype,
                                    const void* grad_out, const void* lse_out, const void* rel,
                                    int64_t emb, void* grad_rel, void* scratch,
                                    size_t scratch_bytes, void* stream);

/* Logsumexp forms. NULL (or beta = 1, eps = 0) is fanin_reduce mode 1. The
 * smoothed form is relmo's LogSumExpAggregation (relmo/models/aggr.py:96-123),
 * the aggregation its models use for "logsumexp":
 *   out[r] = m_r + (1/beta) log(eps + sum over edges j of r of e^(beta (x_j - m_r))),
 *   m_r = max_j x_j (no gradient through it), rows without edges (1/beta) log(eps);
 * its gradient is e^(beta (x_j - out[r])) per edge (the softmax of beta x with
 * the eps term). relmo evaluates it with four ATen passes around a
 * index_reduce_ amax; here it is one planned pass like the plain form. No
 * counterpart in the reference's op library. */
typedef struct relm_mp_lse_form {
   double beta; /* > 0; relmo's default maximum_smoothness is 12 */
   double eps;  /* >= 0; relmo adds 1e-16 */
} relm_mp_lse_form;

/* relm_mp_plan_reduce mode 1 with a logsumexp form (form NULL: plain). */
RELM_MP_API int relm_mp_plan_reduce_lse(const relm_mp_plan* plan, relm_mp_dtype dtype, const relm_mp_lse_form* form,
                                        const void* table, int64_t emb, void* out, void* scratch,
                                        size_t scratch_bytes, void* stream);
/* relm_mp_plan_logsumexp_backward for a form: grad_rel[r] = sum over edges j of
 * r of grad_out[gidx[j]] * e^(beta (rel[r] - lse_out[gidx[j]])). */
RELM_MP_API int relm_mp_plan_logsumexp_backward_ex(const relm_mp_plan* plan, relm_mp_dtype dtype,
                                                   const relm_mp_lse_form* form, const void* grad_out,
                                                   const void* lse_out, const void* rel, int64_t emb,
                                                   void* grad_rel, void* scratch, size_t scratch_bytes,
                                                   void* stream);
/* relm_mp_plan_scatter_logsumexp_backward for a form. */
RELM_MP_API int relm_mp_plan_scatter_logsumexp_backward_ex(const relm_mp_plan* plan, relm_mp_dtype dtype,
                                                           const relm_mp_lse_form* form, const void* grad_out,
                                                           const void* lse_out, const void* rel, int64_t emb,
                                                           const uint32_t* cover, void* grad_rel, void* stream);

/* Sum with a fused epilogue, the indexed sum / mean of the LGAN ops
 * (relmo/ops/mp_common.py:88-118, mp_ops.cpp:3433-3454):
 *   out[r] = base[r] + (sum over edges j of r of table[gidx[j]]) / max(d_r, 1)
 * with d_r = row_div[r] when row_div != NULL (an int64 array over the plan's
 * rows, converted to the value type before the clamp, as
 * `arities.to(dtype).clamp_min(1)`), else the number of edges of r when
 * divide_by_count != 0 (mean), else 1. base may be NULL (0) or equal to out.
 * Scratch: relm_mp_plan_reduce_scratch_bytes(plan, emb, dtype, RELM_MP_MODE_SUM).
 * No counterpart in the reference (its LGAN ops run atomics, then a separate
 * divide pass, cu:938-1026). */
RELM_MP_API int relm_mp_plan_reduce_ex(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* table,
                                       int64_t emb, const void* base, const int64_t* row_div,
                                       int divide_by_count, void* out, void* scratch, size_t scratch_bytes,
                                       void* stream);
/* relm_mp_plan_scatter_rows with each plan row divided by max(row_div[r], 1)
 * (row_div may be NULL). cover may be NULL when every out row is gathered by
 * some edge (nothing is zeroed then): the slot gradient of the LGAN pool,
 * out[s] = table[r] / max(arity[r], 1) through the pool's plan. */
RELM_MP_API int relm_mp_plan_scatter_rows_div(const relm_mp_plan* plan, relm_mp_dtype dtype, const void* table,
                                              int64_t emb, const int64_t* row_div, const uint32_t* cover,
                                              void* out, void* stream);
/* The gather form of the same: out[s] = table[out_index[s]] / max(row_div[out_index[s]], 1)
 * for s < plan->num_edges, where out_index is the array the plan was built from
 * (validated by that build) and the plan gathers the identity (a NULL
 * gather_index: gather_rows == num_edges). Reads the original index order, so
 * slots come out in order with one 16-byte load and store per chunk. */
RELM_MP_API int relm_mp_plan_gather_rows_div(const relm_mp_plan* plan, const int64_t* out_index, relm_mp_dtype dtype,
                                             const void* table, int64_t emb, const int64_t* row_div, void* out,
                                             void* stream);
/* counts[g] = number of the plan's edges gathering row g, g < gather_rows
 * (int32, deterministic integer atomics). */
RELM_MP_API int relm_mp_plan_gather_counts(const relm_mp_plan* plan, int32_t* counts, void* stream);
/* out[r] = in[r] / max(counts[r], 1) for r < rows (out may equal in): the
 * `gathered / counts.clamp_min(1)` of the mean-mode reverse aggregation
 * (mp_ops.cpp:3542-3553). */
RELM_MP_API int relm_mp_divide_rows(relm_mp_dtype dtype, const void* in, int64_t rows, int64_t emb,
                                    const int32_t* counts, void* out, void* stream);

/* ---------------------------------------------------------------------------
 * LGAN ops (`sum` / `mean` modes):
 *
 *   relm_mp_lgan_pool_reduce                  <- lgan_pool_reduce                  (mp_ops.cpp:3350-3469, schema 3778)
 *   relm_mp_lgan_pool_reduce_backward         <- lgan_pool_reduce_backward         (mp_ops.cpp:3471-3572, schema 3781)
 *   relm_mp_lgan_relation_graph_step          <- lgan_relation_graph_step          (mp_ops.cpp:3574-3656, schema 3784)
 *   relm_mp_lgan_relation_graph_step_backward <- lgan_relation_graph_step_backward (mp_ops.cpp:3658-3743, schema 3787)
 *
 * agg(x, src, dst, rows)[t] = sum of x[src[e]] over the edges e with dst[e] = t,
 * divided by max(edges into t, 1) in mode RELM_MP_MODE_MEAN. The relation
 * graph step computes x1 = x + agg(x, rr_src, rr_dst, R), tn = agg(x1, tn_rel,
 * tn_ent, N), nn = agg(x1, nn_rel, nn_ent, N); the pool first forms
 * x[r] = (sum of the slot rows s with slot_to_relation_instance[s] = r) /
 * max(relation_instance_arities[r], 1). Backward ops return the gradient of
 * the first input from the gradients of the three outputs. Each aggregation
 * runs through a plan built in the workspace (one at a time), so every call
 * synchronizes `stream` once per aggregation for index validation.
 * ------------------------------------------------------------------------- */

/* Mode of the LGAN ops, as relmo.ops.mp_constants MODE_MEAN (mode 0 is sum). */
#define RELM_MP_MODE_MEAN 2

typedef struct relm_mp_lgan_graph {
   const int64_t* rr_src; /* relation -> relation edges */
   const int64_t* rr_dst;
   int64_t num_rr;
   const int64_t* tn_rel; /* relation -> entity edges (TN) */
   const int64_t* tn_ent;
   int64_t num_tn;
   const int64_t* nn_rel; /* relation -> entity edges (NN) */
   const int64_t* nn_ent;
   int64_t num_nn;
   int64_t relation_count;  /* R: rows of relation_pair_x (length of relation_instance_arities) */
   int64_t entity_dim_size; /* N: rows of tn_msgs / nn_msgs */
} relm_mp_lgan_graph;

/* One size for all four LGAN entry points (num_slots: rows of slot_messages,
 * 0 for the relation graph step). */
RELM_MP_API size_t relm_mp_lgan_workspace_bytes(const relm_mp_lgan_graph* graph, int64_t num_slots, int64_t emb,
                                                relm_mp_dtype dtype);
RELM_MP_API int relm_mp_lgan_relation_graph_step(relm_mp_dtype dtype, const relm_mp_lgan_graph* graph,
                                                 const void* relation_pair_x, int64_t emb, int mode,
                                                 void* relation_pair_x_out, void* tn_msgs, void* nn_msgs,
                                                 void* workspace, size_t workspace_bytes, void* stream);
RELM_MP_API int relm_mp_lgan_relation_graph_step_backward(relm_mp_dtype dtype, const relm_mp_lgan_graph* graph,
                                                          const void* grad_relation_pair_x,
                                                          const void* grad_tn_msgs, const void* grad_nn_msgs,
                                                          int64_t emb, int mode, void* grad_relation_pair_x_in,
                                                          void* workspace, size_t workspace_bytes, void* stream);
RELM_MP_API int relm_mp_lgan_pool_reduce(relm_mp_dtype dtype, const relm_mp_lgan_graph* graph,
                                         const void* slot_messages, int64_t num_slots, int64_t emb,
                                         const int64_t* slot_to_relation_instance,
                                         const int64_t* relation_instance_arities, int mode,
                                         void* relation_pair_x, void* tn_msgs, void* nn_msgs, void* workspace,
                                         size_t workspace_bytes, void* stream);
RELM_MP_API int relm_mp_lgan_pool_reduce_backward(relm_mp_dtype dtype, const relm_mp_lgan_graph* graph,
                                                  const void* grad_relation_pair_x, const void* grad_tn_msgs,
                                                  const void* grad_nn_msgs, int64_t emb, int64_t num_slots,
                                                  const int64_t* slot_to_relation_instance,
                                                  const int64_t* relation_instance_arities, int mode,
                                                  void* grad_slot_messages, void* workspace,
                                                  size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RELM_MP_H */
