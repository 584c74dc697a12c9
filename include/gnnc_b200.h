/*
 * gnnc_b200.h - C ABI of the B200 runtime for GNNC's GCN / GAT aggregation path.
 *
 * The reference (rdadolf/ml-reentry-mlir, "GNNC") reaches its compiled GCN
 * aggregation through gnnc.execution.run_jit (gnnc/execution/__init__.py:25-69),
 * which JIT-links the MLIR-lowered module and calls it with every CSR input
 * decomposed into (crow_indices, col_indices, values) (gnnc/execution/__init__.py:72-100).
 * The B200 backend replaces that JIT call with the entry points below. A
 * caller binds them through ctypes (Python), cgo, JNI or any FFI that can pass
 * integers and pointers.
 *
 * Conventions
 *  - Every function returns an int status: 0 = GNNC_OK, >0 = gnnc_status_t.
 *    Nothing aborts or traps; the last failure's text is kept per context
 *    (gnnc_last_error).
 *  - Tensor arguments are raw DEVICE pointers (the caller owns them) unless a
 *    parameter says "host". Row strides ("ld*") are in elements.
 *  - Work is issued on the context's stream (gnnc_stream_set); calls return
 *    without synchronising unless stated.
 *  - Index types: CSR row pointers and column indices are int32 on the device
 *    (E < 2^31). The reference uses int64 (posWidth = crdWidth = 64,
 *    test/reference/gcn.raw.mlir:1); the index VALUES are identical.
 *  - One context per device per process; calls on one context are stream
 *    ordered and not thread safe (gnnc/__init__.py:23-30 keeps one MLIR
 *    context per process in the same way).
 */
#ifndef GNNC_B200_H
#define GNNC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GNNC_ABI_VERSION 1

#if defined(__GNUC__)
#define GNNC_API __attribute__((visibility("default")))
#else
#define GNNC_API
#endif

typedef enum gnnc_status {
  GNNC_OK = 0,
  GNNC_ERR_INVALID = 1,     /* bad argument (null pointer, negative size, misaligned stride) */
  GNNC_ERR_UNSUPPORTED = 2, /* valid but not implemented (e.g. too many heads)               */
  GNNC_ERR_CUDA = 3,        /* a CUDA runtime call failed                                      */
  GNNC_ERR_OOM = 4,         /* device allocation failed / workspace too small                 */
  GNNC_ERR_BOUNDS = 5,      /* graph validation found an out-of-range index                   */
  GNNC_ERR_TIMEOUT = 6,     /* a bounded wait gave up                                          */
  GNNC_ERR_NCCL = 7         /* collective failure                                              */
} gnnc_status_t;

typedef enum gnnc_dtype { GNNC_F32 = 0, GNNC_BF16 = 1 } gnnc_dtype_t;

typedef enum gnnc_act { GNNC_ACT_NONE = 0, GNNC_ACT_RELU = 1, GNNC_ACT_ELU = 2 } gnnc_act_t;

typedef struct gnnc_ctx gnnc_ctx_t;
typedef struct gnnc_plan gnnc_plan_t;

/* ------------------------------------------------------------------------ */
/* Context, stream, errors                                                   */
/* ------------------------------------------------------------------------ */

/* Replaces the per-process MLIR context + JIT engine set-up
 * (gnnc/__init__.py:23-39, gnnc/execution/__init__.py:66-68).
 * Allocates the context's small device area and resolves the address of the
 * fixed scratch of gnnc_gat_aggregate_noalloc (loading the library's device
 * code on `device`). */
GNNC_API int gnnc_init(int device, gnnc_ctx_t** out_ctx);
GNNC_API int gnnc_destroy(gnnc_ctx_t* ctx);

/* stream is a cudaStream_t (0 = legacy default stream). */
GNNC_API int gnnc_stream_set(gnnc_ctx_t* ctx, void* stream);

/* Copies the last error text of ctx into buf (NUL terminated, truncated to n). */
GNNC_API int gnnc_last_error(const gnnc_ctx_t* ctx, char* buf, size_t n);
GNNC_API const char* gnnc_status_string(int status);
GNNC_API int gnnc_abi_version(void);

/* Blocks until the context's stream is idle; returns GNNC_ERR_CUDA with the
 * CUDA error text if any earlier launch failed. */
GNNC_API int gnnc_synchronize(gnnc_ctx_t* ctx);

/* Scratch memory. The library grows an internal device workspace on demand;
 * a caller may instead bind its own buffer (it must outlive every call that
 * uses it). workspace_query returns the bytes a GAT / softmax aggregation of
 * feature width F needs with this plan. */
GNNC_API int gnnc_workspace_query(gnnc_ctx_t* ctx, const gnnc_plan_t* plan, int64_t F, size_t* bytes);
GNNC_API int gnnc_workspace_bind(gnnc_ctx_t* ctx, void* ptr, size_t bytes);

/* ------------------------------------------------------------------------ */
/* Graph preparation                                                         */
/* ------------------------------------------------------------------------ */

/* COO edge list -> CSR by destination, columns (sources) ascending within a
 * row. Replaces normalized_csr_adj's flip + coalesce + to_sparse_csr
 * (gnnc/examples/util.py:16-41) and GATConv's remove_self_loops +
 * add_self_loops (PyG GATConv.forward, called from
 * experiments/pyg-baseline/run.py:78-88).
 *   src, dst      : int64 [E] (edge_index[0], edge_index[1]); device
 *   self_loops    : 1 = drop every (i,i) edge and add exactly one per node
 *                   (PyG add_remaining_self_loops with unit weights, and
 *                   remove_self_loops + add_self_loops)
 *   dedupe        : 1 = merge duplicate (dst,src) pairs like coalesce();
 *                   mult[k] receives how many input edges entry k merged.
 *                   0 = keep duplicates (GATConv treats each as its own edge).
 *   rowptr        : int32 [N+1]; col : int32 [capacity]; mult : int32 [capacity]
 *                   or NULL; capacity >= E + N when self_loops, else >= E
 *   E_out         : host; number of CSR entries written
 * Indices outside [0,N) return GNNC_ERR_BOUNDS and write nothing useful.
 * Blocks the calling thread until E_out is known. */
GNNC_API int gnnc_csr_from_coo(gnnc_ctx_t* ctx, const int64_t* src, const int64_t* dst, int64_t E,
                      int64_t N, int self_loops, int dedupe, int32_t* rowptr, int32_t* col,
                      int32_t* mult, int64_t capacity, int64_t* E_out);

/* GCN symmetric normalisation over a CSR built by gnnc_csr_from_coo(self_loops=1).
 * Columns outside [0, N) get weight 0.
 * Restates PyG gcn_norm as called at gnnc/examples/util.py:22:
 *   deg[d]  = number of input edges into d (mult-weighted, self-loop included)
 *   dinv[d] = 1/sqrt(deg[d]) (IEEE-rounded sqrt then divide; inf -> 0)
 *   w[k]    = sum over the mult[k] merged copies of dinv[src]*dinv[dst]
 * Bit-identical to torch CPU for deg < 2^24. mult may be NULL (all 1).
 * deg and dinv may be NULL. */
GNNC_API int gnnc_gcn_norm(gnnc_ctx_t* ctx, const int32_t* rowptr, const int32_t* col,
                  const int32_t* mult, int64_t N, float* deg, float* dinv, float* w);

/* Checks rowptr[0] >= 0, rowptr non-decreasing, rowptr[n_rows] <= E and
 * every col in [0, n_src). Returns GNNC_ERR_BOUNDS (with the first bad
 * position in the error text) when not. Synchronous. */
/* Mean-aggregation weights of SAGEConv on a CSR adjacency:
 *   w_out[k] = w_in[k] / max(#{j in row(k) : w_in[j] != 0}, 1)
 * (w_in NULL: unit weights, every stored edge counted). Restates the
 * `_sparse_mm.reduce("mean")` rewrite (A.X) / clamp_min(row_nnz, 1)
 * (gnnc/conversion/tm_tensor_to_torch/despecialize_sparse_mm_reduce.py:1-75)
 * as weights on the edges, so gnnc_sage_aggregate is a weighted SpMM. */
GNNC_API int gnnc_mean_norm(gnnc_ctx_t* ctx, const int32_t* rowptr, int64_t n_rows,
                            const float* w_in, float* w_out);

GNNC_API int gnnc_csr_validate(gnnc_ctx_t* ctx, const int32_t* rowptr, const int32_t* col,
                      int64_t n_rows, int64_t E, int64_t n_src);

/* ------------------------------------------------------------------------ */
/* Aggregation plan (degree-skew split)                                      */
/* ------------------------------------------------------------------------ */

/* Builds the row schedule for one CSR: rows of degree <= cta_threshold are
 * processed by one warp each; longer rows by a whole CTA; rows longer than
 * split_threshold are cut into segments of at most split_threshold edges
 * processed by separate CTAs and combined by a merge step. The plan depends
 * only on rowptr (device, n_rows+1 entries) and is reused across layers and
 * calls. 0 selects the defaults: cta_threshold 256 (launches on 256-wide
 * rows give rows of up to 1024 edges to the warp path), split_threshold
 * max(4096, edges / (2 * SMs * 4)), so a row is split only when it is a
 * sizeable share of the launch. Replaces the survey's gnnc_row_split_plan.
 * Synchronous (reads rowptr back once). */
GNNC_API int gnnc_plan_create(gnnc_ctx_t* ctx, const int32_t* rowptr, int64_t n_rows,
                     int32_t cta_threshold, int32_t split_threshold, gnnc_plan_t** out_plan);
GNNC_API int gnnc_plan_destroy(gnnc_plan_t* plan);
/* info[0..5] = n_rows, n_warp_rows, n_cta_rows, n_split_rows, n_segments, max_degree */
GNNC_API int gnnc_plan_info(const gnnc_plan_t* plan, int64_t* info6);

/* ------------------------------------------------------------------------ */
/* Dense projection                                                          */
/* ------------------------------------------------------------------------ */

/* h[N,F] = x[N,K] . w[F,K]^T (nn.Linear weight layout, no bias), fp32
 * accumulation; optionally the per-head attention coefficients of GATConv:
 *   asrc[n,hd] = sum_c h[n,hd*C+c] * att_src[hd*C+c]    (H heads, C = F/H)
 *   adst[n,hd] = sum_c h[n,hd*C+c] * att_dst[hd*C+c]
 * computed from the fp32 accumulator. Replaces aten.linear + view + mul + sum
 * (experiments/gatconv/dumps/gat.1-raw-torch.mlir:5-24) and the dense
 * linalg.matmul X.W^T (test/reference/gcn.linalg-on-tensors.mlir:19).
 *   x_dtype   : dtype of x and w (GNNC_F32 or GNNC_BF16)
 *   h_dtype   : dtype of h
 *   att_src/att_dst/asrc/adst : NULL when not wanted (all four or none)
 * Strides ldx, ldw, ldh in elements; rows must start 16-byte aligned. */
GNNC_API int gnnc_proj(gnnc_ctx_t* ctx, const void* x, int x_dtype, int64_t ldx, const void* w,
              int64_t ldw, int64_t N, int64_t K, int64_t F, const float* att_src,
              const float* att_dst, int64_t H, void* h, int h_dtype, int64_t ldh, float* asrc,
              float* adst);

/* ------------------------------------------------------------------------ */
/* Aggregation (the hot path)                                                */
/* ------------------------------------------------------------------------ */
/* Shared arguments:
 *   plan        : from gnnc_plan_create on the same rowptr (edge ranges are
 *                 clamped to the planned [rowptr[0], rowptr[n_rows]))
 *   rowptr,col  : CSR by destination: rows [0,n_rows), col = source row of h;
 *                 col (and w / s) must hold rowptr[n_rows] entries. A column
 *                 outside [0, n_src) is skipped and reported as
 *                 GNNC_ERR_BOUNDS by the next gnnc_synchronize.
 *   h           : [n_src, F] feature table, row stride ldh, dtype h_dtype
 *   bias        : [F_out] fp32 or NULL; act: gnnc_act_t applied after bias
 *   log_softmax : 1 = row-wise log_softmax after bias/act (final layer)
 *   out         : [n_rows, F_out] row stride ldo, dtype out_dtype
 */

/* GCNConv aggregation on a pre-normalised CSR: out = A.h (+bias, act, ...).
 * Replaces aten._sparse_mm(A_csr, H) (test/reference/gcn.raw.mlir:7,13),
 * rewritten to aten.mm by gnnc/conversion/tm_tensor_to_torch/despecialize_sparse_mm.py:15-25
 * and lowered to the sparsifier's CSR row loop (gnnc/schedule/sparse.py:47-62).
 *   w : fp32 [E] edge values (CSR values). F_out = F. */
GNNC_API int gnnc_gcn_aggregate(gnnc_ctx_t* ctx, const gnnc_plan_t* plan, const int32_t* rowptr,
                       const int32_t* col, const float* w, const void* h, int h_dtype,
                       int64_t ldh, int64_t n_rows, int64_t n_src, int64_t F, const float* bias,
                       int act, int log_softmax, void* out, int out_dtype, int64_t ldo);

/* SAGEConv (mean aggregation, root weight) after its two projections
 * h = x.W_l^T and root = x.W_r^T:  out = A_mean.h + root + bias, then act /
 * log_softmax. w holds gnnc_mean_norm weights. Replaces the SAGE layer of
 * test/reference/sage.raw.mlir:5-14 (_sparse_mm.reduce "mean", linear with
 * bias, linear without bias, add, relu); root [n_rows, F] row stride ldr,
 * dtype root_dtype, indexed like out. */
GNNC_API int gnnc_sage_aggregate(gnnc_ctx_t* ctx, const gnnc_plan_t* plan, const int32_t* rowptr,
                        const int32_t* col, const float* w, const void* h, int h_dtype,
                        int64_t ldh, const void* root, int root_dtype, int64_t ldr,
                        int64_t n_rows, int64_t n_src, int64_t F, const float* bias, int act,
                        int log_softmax, void* out, int out_dtype, int64_t ldo);

/* One fused GATConv layer after the projection:
 *   e_k   = LeakyReLU_slope(asrc[src_k,hd] + adst[row,hd])
 *   a_k   = exp(e_k - max_row e) / (sum_row exp(e - max) + 1e-16)
 *   out   = sum_k a_k * h[src_k]  ->  concat heads [H*C] or mean over heads [C]
 * Replaces the PyG eager chain at experiments/gatconv/dumps/gat.1-raw-torch.mlir:25-129
 * (index_select x2, add, leaky_relu, scatter_reduce amax, exp, scatter_add,
 * +1e-16, div, gather * alpha, scatter_add). Logits never reach HBM.
 *   asrc : [n_src, H] fp32; adst : [n_rows, H] fp32 (row-local)
 *   F = H*C; F_out = concat ? H*C : C. H <= 16. */
GNNC_API int gnnc_gat_aggregate(gnnc_ctx_t* ctx, const gnnc_plan_t* plan, const int32_t* rowptr,
                       const int32_t* col, const void* h, int h_dtype, int64_t ldh,
                       const float* asrc, const float* adst, int64_t n_rows, int64_t n_src,
                       int64_t H, int64_t C, float negative_slope, int concat, const float* bias,
                       int act, int log_softmax, void* out, int out_dtype, int64_t ldo);

/* Edge softmax over given per-edge scores followed by the weighted SpMM:
 *   out[row] = sum_k exp(s_k - max) / (sum exp(s - max) + eps) * h[src_k]
 * s : fp32 [E, H] in CSR order. The core of the GAT chain without the
 * SDDMM; eps = 0 reproduces experiments/gat-gpu-codegen/gat-kernel.mlir:31-132,
 * eps = 1e-16 reproduces PyG utils.softmax. */
GNNC_API int gnnc_softmax_aggregate(gnnc_ctx_t* ctx, const gnnc_plan_t* plan, const int32_t* rowptr,
                           const int32_t* col, const float* s, const void* h, int h_dtype,
                           int64_t ldh, int64_t n_rows, int64_t n_src, int64_t H, int64_t C,
                           float eps, int concat, const float* bias, int act, int log_softmax,
                           void* out, int out_dtype, int64_t ldo);

/* gnnc_gat_aggregate for callers that must not allocate device memory.
 * This entry point has no counterpart in the reference.
 * Who needs it: a serving process that reserves its whole memory budget at
 * start-up (a cudaMalloc in the middle of a request can fail because the
 * device is already full, and cudaMalloc / cudaFree synchronise the device),
 * or a host runtime that owns all device memory through its own pool and
 * forbids libraries from allocating behind its back. gnnc_gat_aggregate may
 * grow the context workspace with cudaMalloc; this variant never calls
 * cudaMalloc, cudaFree or any allocating routine.
 * Same arguments and results as gnnc_gat_aggregate. Its scratch (work
 * counters, the bad-index flag, split-row partials) is one fixed 16 MiB device
 * array inside the library, held by every GPU that loads the library until
 * the process exits. A plan whose split rows need more than 16 MiB - 256 B of
 * partials (n_segments * (32 + F_pad) * 4 bytes) is rejected with
 * GNNC_ERR_UNSUPPORTED before anything is launched.
 * gnnc_init looks up the array's device address for its context (that device
 * current). With CUDA's lazy module loading that lookup is what loads this
 * library's device code on the device and reserves the 16 MiB, so any
 * allocation happens in gnnc_init and never in this entry point. The address
 * belongs to the context: after cudaDeviceReset (which also frees the
 * context's own buffers) make a new context. All calls on a device share the
 * one array, which keeps the last call's contents (the counters are cleared
 * by each call): calls that overlap on the GPU (different streams or contexts
 * of the same device) race and give wrong results; serialise them. */
GNNC_API int gnnc_gat_aggregate_noalloc(gnnc_ctx_t* ctx, const gnnc_plan_t* plan,
                                        const int32_t* rowptr, const int32_t* col, const void* h,
                                        int h_dtype, int64_t ldh, const float* asrc,
                                        const float* adst, int64_t n_rows, int64_t n_src,
                                        int64_t H, int64_t C, float negative_slope, int concat,
                                        const float* bias, int act, int log_softmax, void* out,
                                        int out_dtype, int64_t ldo);

/* ------------------------------------------------------------------------ */
/* Peer memory (multi-GPU exchange read straight from the owner's HBM)       */
/* ------------------------------------------------------------------------ */
/* The reference has no multi-GPU path (internal-docs/project-summary.md:105);
 * these replace nothing there. With one process per GPU, a rank exports the
 * device buffer holding the rows it owns and every other rank maps it, so the
 * projection reads remote input rows over NVLink inside its own tile loads
 * (TMA without multicast) instead of after an all-gather.
 *   gnnc_peer_export : handle (GNNC_PEER_HANDLE_BYTES bytes, opaque, to be sent
 *                      to the other ranks) and the offset of ptr inside its
 *                      allocation; ptr must lie in a cudaMalloc allocation of
 *                      ctx's device (GNNC_ERR_INVALID / GNNC_ERR_CUDA otherwise)
 *   gnnc_peer_open   : maps another process's exported buffer into ctx's
 *                      device; *ptr = the exported ptr's address here
 *   gnnc_peer_copy   : bytes from src to dst on ctx's stream, either side a
 *                      mapping (a copy-engine transfer; no SM is used)
 *   gnnc_peer_close  : unmaps (ptr and offset as returned / passed to open)
 * The exporter keeps its buffer alive until every importer has closed it, and
 * the ranks order writes and reads of the buffer themselves (e.g. a
 * stream-ordered collective between writing and reading). */
#define GNNC_PEER_HANDLE_BYTES 64
GNNC_API int gnnc_peer_export(gnnc_ctx_t* ctx, const void* ptr, void* handle, uint64_t* offset);
GNNC_API int gnnc_peer_open(gnnc_ctx_t* ctx, const void* handle, uint64_t offset, void** ptr);
GNNC_API int gnnc_peer_copy(gnnc_ctx_t* ctx, void* dst, const void* src, size_t bytes);
GNNC_API int gnnc_peer_close(gnnc_ctx_t* ctx, void* ptr, uint64_t offset);

/* dst[i] = src[idx[i]] for i < n: rows of row_bytes bytes, strides in bytes,
 * all 16-byte aligned. Packs the rows another rank needs into one contiguous
 * block that it then pulls with one gnnc_peer_copy. An index outside
 * [0, n_src) leaves its row untouched and is reported as GNNC_ERR_BOUNDS by
 * the next gnnc_synchronize. No reference counterpart (multi-GPU exchange). */
GNNC_API int gnnc_gather_rows(gnnc_ctx_t* ctx, const void* src, int64_t ld_src,
                              const int32_t* idx, int64_t n, int64_t n_src, void* dst,
                              int64_t ld_dst, int64_t row_bytes);

/* Diagnostics; no counterpart in the reference. Every wait of the tensor-core
 * projection on its pipeline (mbarriers) gives up after 2 s of %globaltimer,
 * raises an abort flag, drains its copies / MMAs and frees TMEM, and
 * gnnc_synchronize then returns GNNC_ERR_TIMEOUT. gnnc_wait_selftest runs that
 * same bounded wait on an mbarrier that nothing arrives on (nothing else in
 * flight), with a limit of limit_ns (0 < limit_ns <= 2e9), on ctx's stream:
 * the next gnnc_synchronize returns GNNC_ERR_TIMEOUT and clears the report,
 * and the context stays usable. */
GNNC_API int gnnc_wait_selftest(gnnc_ctx_t* ctx, int64_t limit_ns);

/* One NCCL communicator per context, for the exchange step of a
 * destination-row partition (replaces the reference-side all-gather a
 * partitioned layer needs; the reference itself has no multi-GPU path,
 * internal-docs/project-summary.md:105):
 *   gnnc_comm_unique_id : rank 0 makes the id (GNNC_COMM_ID_BYTES bytes) and
 *                         hands it to the other ranks by any host means
 *   gnnc_comm_init      : joins communicator `id` as `rank` of `nranks` on
 *                         ctx's device, waiting at most 120 s for every rank
 *   gnnc_comm_init_timeout : the same with a deadline of timeout_ms: if not
 *                         every rank has joined by then, the communicator is
 *                         aborted and GNNC_ERR_TIMEOUT returned (the context
 *                         stays usable and may join another communicator)
 *   gnnc_allgather      : recvbuf[r*count .. (r+1)*count) = rank r's sendbuf
 *                         (count elements of dtype GNNC_F32 or GNNC_BF16), on
 *                         ctx's stream
 *   gnnc_comm_wait      : waits at most timeout_ms for ctx's stream (its
 *                         collectives included); a collective that cannot
 *                         finish (a peer died between steps) aborts the
 *                         communicator and returns GNNC_ERR_TIMEOUT, an
 *                         asynchronous NCCL error returns GNNC_ERR_NCCL
 *   gnnc_comm_destroy   : waits for ctx's stream, destroys the communicator
 *                         (gnnc_destroy also does)
 * Communicators are non-blocking (ncclConfig_t.blocking = 0): the host polls
 * their state against the deadlines instead of blocking inside NCCL. NCCL is
 * loaded on first use (the copy already in the process, else libnccl.so.2);
 * failures return GNNC_ERR_NCCL with NCCL's message. */
#define GNNC_COMM_ID_BYTES 128
GNNC_API int gnnc_comm_unique_id(gnnc_ctx_t* ctx, void* id);
GNNC_API int gnnc_comm_init(gnnc_ctx_t* ctx, const void* id, int rank, int nranks);
GNNC_API int gnnc_comm_init_timeout(gnnc_ctx_t* ctx, const void* id, int rank, int nranks,
                                    int64_t timeout_ms);
GNNC_API int gnnc_allgather(gnnc_ctx_t* ctx, const void* sendbuf, void* recvbuf, size_t count,
                            int dtype);
GNNC_API int gnnc_comm_wait(gnnc_ctx_t* ctx, int64_t timeout_ms);
GNNC_API int gnnc_comm_destroy(gnnc_ctx_t* ctx);

#ifdef __cplusplus
}
#endif

#endif /* GNNC_B200_H */
