/*
 * projectai_cuda.h — C ABI of libprojectai_cuda.so, the B200 (sm_100a) compute backend that plugs in
 * behind project-ai's IComputeBackend seam.
 *
 * Every entry point here is what a P/Invoke layer for ProjectAI.Core/IComputeBackend.cs would bind:
 * plain pointers, sizes and a POD tensor descriptor, no C++ or torch types. Each declaration names the
 * reference member it replaces (file:line, paths relative to the project-ai repository).
 *
 * Conventions
 *  - Every function returns a pai_status; on failure pai_last_error() holds a message for the calling thread.
 *    The status maps onto the .NET exception the reference throws for the same condition:
 *      PAI_ERR_ARGUMENT      -> ArgumentException            (shape / rank / broadcast mismatch)
 *      PAI_ERR_OUT_OF_RANGE  -> ArgumentOutOfRangeException  (axis, id or target out of range)
 *      PAI_ERR_INVALID_OP    -> InvalidOperationException
 *      PAI_ERR_OUT_OF_MEMORY -> OutOfMemory; the message always contains "out of memory"
 *                               (ProjectAI.Trainer/Program.cs:152-157 matches on that text)
 *  - Ops never modify their inputs. Each op allocates a fresh, contiguous, zero-offset result in the
 *    context's current scope and describes it in *out (IComputeBackend.cs:9-96: "every op consumes and
 *    produces Tensor handles allocated by the same backend"). Inputs may be arbitrary views: element
 *    strides (0 = broadcast), a non-zero element offset, rank <= PAI_MAX_RANK.
 *  - All work is ordered on the context's compute stream. Only pai_to_host, pai_sync and the ops that
 *    return a host scalar block the caller.
 *  - dtype: the hot path computes in F32 (the CPU oracle is F32-only, CpuComputeBackend.cs:41-53).
 */
#ifndef PROJECTAI_CUDA_H
#define PROJECTAI_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PAI_MAX_RANK 8

/* ProjectAI.Core/DType.cs:4-13, same order. */
enum pai_dtype { PAI_F32 = 0, PAI_F16 = 1, PAI_BF16 = 2, PAI_I64 = 3, PAI_I32 = 4, PAI_U8 = 5, PAI_BOOL = 6 };

typedef enum pai_status {
  PAI_OK = 0,
  PAI_ERR_ARGUMENT = 1,
  PAI_ERR_OUT_OF_RANGE = 2,
  PAI_ERR_INVALID_OP = 3,
  PAI_ERR_OUT_OF_MEMORY = 4,
  PAI_ERR_CUDA = 5,
  PAI_ERR_NCCL = 6,
  PAI_ERR_TIMEOUT = 7,
  PAI_ERR_UNSUPPORTED = 8,
  PAI_ERR_IO = 9,           /* IOException / FileNotFoundException: a file could not be opened, read or written */
  PAI_ERR_INVALID_DATA = 10 /* InvalidDataException: a checkpoint or dataset file is malformed */
} pai_status;

/* A tensor view (ProjectAI.Core/Tensor.cs:17-48): storage base + element offset + shape + element strides.
 * `base` is the pointer returned by an allocating call; views share it. */
typedef struct pai_tensor {
  void* base;
  int64_t offset;
  int32_t rank;
  int32_t dtype;
  int32_t dims[PAI_MAX_RANK];
  int64_t strides[PAI_MAX_RANK];
} pai_tensor;

/* One backend instance bound to one device and one compute stream (IComputeBackend.cs:9-12). */
typedef struct pai_ctx pai_ctx;

/* Thread-local message for the last failing call on this thread. Never NULL. */
const char* pai_last_error(void);

/* ---- Lifetime (IComputeBackend.cs:9 IDisposable; Backends.cs:24-31 factory) ---- */
pai_status pai_ctx_create(int device_ordinal, pai_ctx** out);
pai_status pai_ctx_destroy(pai_ctx* ctx);
pai_status pai_sync(pai_ctx* ctx);
/* Device name, for IComputeBackend.Name / Device (IComputeBackend.cs:11-12). */
pai_status pai_device_name(pai_ctx* ctx, char* buf, int32_t buf_len);

/* ---- Allocation & host transfer (IComputeBackend.cs:15-18; CpuComputeBackend.cs:41-81) ---- */
/* Allocate: zero-filled contiguous tensor (CpuComputeBackend.cs:41-42 returns a zeroed array). */
pai_status pai_alloc(pai_ctx* ctx, int32_t rank, const int32_t* dims, int32_t dtype, pai_tensor* out);
/* FromHost: `count` floats, row-major, must equal the shape's element count. */
pai_status pai_from_host(pai_ctx* ctx, const float* host, int64_t count, int32_t rank, const int32_t* dims,
                         int32_t dtype, pai_tensor* out);
/* ToHost: the view's logical elements in row-major order (CpuComputeBackend.cs:55-67). Blocks. */
pai_status pai_to_host(pai_ctx* ctx, const pai_tensor* src, float* host, int64_t count);
/* Copy: logical elements of src into a (possibly strided) destination view of equal element count
 * (CpuComputeBackend.cs:69-81). */
pai_status pai_copy(pai_ctx* ctx, const pai_tensor* src, const pai_tensor* dst);

/* ---- Scopes (IComputeBackend.cs:69-95; semantics of TorchComputeBackend.cs:208-218) ----
 * scope_begin pushes a scope; every allocation lands in the innermost open scope (or in no scope).
 * scope_end frees everything the innermost scope owns except blocks passed to keep_alive, which move to
 * the enclosing scope (exactly one level) or to no scope.
 * release frees a block now (a superseded moment or gradient).
 * finalize is the garbage-collector path: it frees a block only if no open scope owns it. */
pai_status pai_scope_begin(pai_ctx* ctx);
pai_status pai_scope_end(pai_ctx* ctx);
pai_status pai_keep_alive(pai_ctx* ctx, const void* base);
pai_status pai_release(pai_ctx* ctx, const void* base);
pai_status pai_finalize(pai_ctx* ctx, const void* base);
/* Bytes currently allocated to tensors, the peak since the last reset, and bytes held by the caching
 * allocator (in use + cached). */
pai_status pai_memory_stats(pai_ctx* ctx, int64_t* in_use, int64_t* peak, int64_t* reserved);
pai_status pai_reset_peak(pai_ctx* ctx);

/* ---- Elementwise, NumPy broadcasting (IComputeBackend.cs:20-31; CpuComputeBackend.cs:86-156, 304-317) ---- */
pai_status pai_add(pai_ctx* ctx, const pai_tensor* a, const pai_tensor* b, pai_tensor* out);
pai_status pai_sub(pai_ctx* ctx, const pai_tensor* a, const pai_tensor* b, pai_tensor* out);
pai_status pai_mul(pai_ctx* ctx, const pai_tensor* a, const pai_tensor* b, pai_tensor* out);
pai_status pai_div(pai_ctx* ctx, const pai_tensor* a, const pai_tensor* b, pai_tensor* out);
pai_status pai_add_scalar(pai_ctx* ctx, const pai_tensor* a, float scalar, pai_tensor* out);
pai_status pai_mul_scalar(pai_ctx* ctx, const pai_tensor* a, float scalar, pai_tensor* out);
pai_status pai_sqrt(pai_ctx* ctx, const pai_tensor* x, pai_tensor* out);
pai_status pai_sigmoid(pai_ctx* ctx, const pai_tensor* x, pai_tensor* out);

/* ---- Linear algebra (IComputeBackend.cs:33-35; CpuComputeBackend.cs:159-219) ----
 * Batched GEMM over the trailing two axes with NumPy batch broadcasting; transpose_b != 0 treats b's
 * trailing axes as [n, k]. Computed with a 3xTF32 split on the tcgen05 tensor cores. */
pai_status pai_matmul(pai_ctx* ctx, const pai_tensor* a, const pai_tensor* b, int32_t transpose_b, pai_tensor* out);

/* ---- Reductions along one axis (IComputeBackend.cs:37-43; CpuComputeBackend.cs:248-301) ---- */
pai_status pai_sum(pai_ctx* ctx, const pai_tensor* x, int32_t axis, int32_t keep_dims, pai_tensor* out);
pai_status pai_mean(pai_ctx* ctx, const pai_tensor* x, int32_t axis, int32_t keep_dims, pai_tensor* out);
pai_status pai_max(pai_ctx* ctx, const pai_tensor* x, int32_t axis, int32_t keep_dims, pai_tensor* out);
/* Index of the largest entry of each row of a [rows..., n] view (last axis unit-stride, leading axes collapsing to
 * one row stride), as float indices in a new [rows] tensor, with the rules of ArgMax (ProjectAI.Models/Sampling.cs:
 * 15-31, used by GreedySampler, :33-38): NaN entries are skipped, ties resolve to the lowest index, and a row without
 * a number gives 0. Greedy decoding then reads one index per sequence instead of each sequence's logits row. */
pai_status pai_argmax_rows(pai_ctx* ctx, const pai_tensor* x, pai_tensor* out);

/* ---- Transformer primitives (IComputeBackend.cs:45-49; CpuComputeBackend.cs:322-420) ---- */
pai_status pai_softmax(pai_ctx* ctx, const pai_tensor* x, int32_t axis, pai_tensor* out);
pai_status pai_rmsnorm(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* weight, float eps, pai_tensor* out);
pai_status pai_silu(pai_ctx* ctx, const pai_tensor* x, pai_tensor* out);
pai_status pai_rotary(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* cos, const pai_tensor* sin, pai_tensor* out);

/* ---- Indexing & loss (IComputeBackend.cs:51-59; CpuComputeBackend.cs:424-500) ----
 * ids / targets are host int32 arrays, as the contract's int[] parameters are. */
pai_status pai_gather(pai_ctx* ctx, const pai_tensor* table, const int32_t* ids, int64_t n_ids, pai_tensor* out);
pai_status pai_scatter_add_rows(pai_ctx* ctx, const pai_tensor* rows, const int32_t* ids, int64_t n_ids,
                                int32_t row_count, pai_tensor* out);
pai_status pai_cross_entropy(pai_ctx* ctx, const pai_tensor* logits, const int32_t* targets, int64_t n_targets,
                             int32_t ignore_index, pai_tensor* out);
pai_status pai_cross_entropy_grad(pai_ctx* ctx, const pai_tensor* logits, const int32_t* targets, int64_t n_targets,
                                  int32_t ignore_index, pai_tensor* out);

/* ---- Structural (IComputeBackend.cs:61-68; CpuComputeBackend.cs:509-540) ---- */
pai_status pai_cat(pai_ctx* ctx, const pai_tensor* a, const pai_tensor* b, int32_t axis, pai_tensor* out);

/* ==== Fused extensions ====
 * Optional ops that a backend may offer beyond the reference seam. The reference composes each of them
 * from the primitives above; a caller that finds them absent composes them the same way. */

/* Causal scaled-dot-product attention with GQA, replacing the composed chain of
 * ProjectAI.Models/Modules.cs:169-196 (Contiguous q/k/v, scores = (q*scale)·kᵀ, + causal mask, softmax, ·v).
 * q [B,H,S,D], k/v [B,KVH,L,D] (any strides), H % KVH == 0; query i sits at absolute position
 * pos_offset + i and attends keys j <= pos_offset + i when causal != 0 (Modules.cs:211-218).
 * out: [B,S,H,D] contiguous (the merged-heads layout of Modules.cs:199-200);
 * lse: [B,H,S] row log-sum-exp (natural log) of the scaled, masked scores, kept for the backward. */
pai_status pai_sdpa_fwd(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k, const pai_tensor* v, float scale,
                        int32_t causal, int32_t pos_offset, pai_tensor* out, pai_tensor* lse);
/* Gradients of pai_sdpa_fwd (the Autograd.cs:54-73 MatMul and :197-205 Softmax rules fused).
 * dout is [B,S,H,D] (any strides); dq [B,H,S,D], dk/dv [B,KVH,L,D] contiguous (GQA groups summed). */
pai_status pai_sdpa_bwd(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k, const pai_tensor* v,
                        const pai_tensor* out, const pai_tensor* lse, const pai_tensor* dout, float scale,
                        int32_t causal, int32_t pos_offset, pai_tensor* dq, pai_tensor* dk, pai_tensor* dv);
/* RMSNorm backward (Autograd.cs:223-244): dx and dw = Σ_rows g⊙x·inv in one pass over x and g. */
pai_status pai_rmsnorm_bwd(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* weight, const pai_tensor* g,
                           float eps, pai_tensor* dx, pai_tensor* dw);
/* SwiGLU gate: silu(gate) ⊙ up (Modules.cs:103-108 with Autograd.cs:208-217 and the Mul rule). */
pai_status pai_silu_mul_fwd(pai_ctx* ctx, const pai_tensor* gate, const pai_tensor* up, pai_tensor* out);
pai_status pai_silu_mul_bwd(pai_ctx* ctx, const pai_tensor* gate, const pai_tensor* up, const pai_tensor* g,
                            pai_tensor* dgate, pai_tensor* dup);
/* Cross-entropy value and gradient in one read of the logits (CpuComputeBackend.cs:453-500 fused with
 * Autograd.cs:187-192). loss: scalar tensor. grad = (softmax − onehot)/count · grad_scale. */
pai_status pai_cross_entropy_fused(pai_ctx* ctx, const pai_tensor* logits, const int32_t* targets, int64_t n_targets,
                                   int32_t ignore_index, float grad_scale, pai_tensor* loss, pai_tensor* grad);
/* One AdamW update in place on p, m, v (ProjectAI.Core/Optimizers.cs:81-123 in one pass, same operation
 * order per element). p, g, m, v: contiguous tensors of equal element count. grad_scale multiplies g
 * first (1/world for a data-parallel sum). */
pai_status pai_adamw_step(pai_ctx* ctx, const pai_tensor* p, const pai_tensor* g, const pai_tensor* m,
                          const pai_tensor* v, float lr, float beta1, float beta2, float eps, float weight_decay,
                          int32_t t, float grad_scale);

/* RMSNorm backward that allocates nothing: no counterpart in the reference. It is for callers that cannot call
 * cudaMalloc, such as a process that reserves all device memory for its own pools, or code that must avoid the
 * synchronisation an allocation can cause. The caller passes dense F32 inputs and dense F32 outputs: dx shaped
 * like x, dw shaped [d]. The per-block partial sums live in a fixed 4 MiB file-scope device array that every GPU
 * loading the library holds until exit. The first call on a device resolves that array's address
 * (cudaGetSymbolAddress), so make it before any stream capture. Calls share the array: calls that overlap on the
 * GPU race, while calls ordered on one stream are safe. Rows longer than 8192 elements are rejected with
 * PAI_ERR_OUT_OF_RANGE. Results match pai_rmsnorm_bwd within float rounding (1e-4): the dw partials are summed in
 * a different order, so the two are not bit-identical. */
pai_status pai_rmsnorm_bwd_noalloc(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* weight, const pai_tensor* g,
                                   float eps, const pai_tensor* dx, const pai_tensor* dw);

/* ==== KV-cache decode as a replayed CUDA graph (no counterpart in the reference) ====
 * Consecutive decode steps (ProjectAI.Training/Inference.cs:46-56 feeding Modules.cs:142-204 and the cache of
 * Modules.cs:290-370) differ only in their token ids and their position. These entry points are the decode-step ops
 * with both read from device tensors, so one captured step replays for every later token: `ids` holds token ids
 * and `pos` (one element) the position of the first new query row, both as integral F32 values written with
 * pai_write before each replay. A value out of range cannot raise on the device: the kernel sets the device
 * error flag (pai_check_device_error) and skips the work, and callers validate ids and positions on the host. */
typedef struct pai_graph pai_graph;
/* Host -> device copy into an existing dense tensor (stream-ordered; the host buffer may be reused on return). */
pai_status pai_write(pai_ctx* ctx, const float* host, int64_t count, const pai_tensor* dst);
/* Gather (IComputeBackend.cs:51-53) with ids from a device tensor: out = table rows ids, shape ids.shape + [d]. */
pai_status pai_gather_dev(pai_ctx* ctx, const pai_tensor* table, const pai_tensor* ids, pai_tensor* out);
/* RotaryEmbedding (IComputeBackend.cs:49) of x [..., S, d] at positions pos .. pos+S-1 of full [T, d] tables. */
pai_status pai_rotary_at(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* cos_table, const pai_tensor* sin_table,
                         const pai_tensor* pos, pai_tensor* out);
/* Writes k, v [B, KVH, S, D] into positions pos .. pos+S-1 of the caches [B, KVH, T, D] (the KvCache append). */
pai_status pai_kv_append(pai_ctx* ctx, const pai_tensor* k, const pai_tensor* v, const pai_tensor* k_cache,
                         const pai_tensor* v_cache, const pai_tensor* pos);
/* pai_rotary_at of q into q_out and of k into cache positions pos .. pos+S-1, with v copied there: the rotations and
 * the cache append of one decode step in one launch (values identical to pai_rotary_at + pai_kv_append). */
pai_status pai_rope_append(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k, const pai_tensor* v,
                           const pai_tensor* cos_table, const pai_tensor* sin_table, const pai_tensor* k_cache,
                           const pai_tensor* v_cache, const pai_tensor* pos, pai_tensor* q_out);
/* pai_rope_append followed by pai_sdpa_decode on its results, in one launch: q, k and v [B, heads, S, D] arrive
 * unrotated (e.g. views of the fused q|k|v product); the rotated keys and the values are written into the caches at
 * positions pos .. pos+S-1 and out [B, S, H, D] holds the causal attention over positions 0 .. pos+S-1. */
pai_status pai_attn_decode_step(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k, const pai_tensor* v,
                                const pai_tensor* cos_table, const pai_tensor* sin_table, const pai_tensor* k_cache,
                                const pai_tensor* v_cache, const pai_tensor* pos, float scale, pai_tensor* out);
/* Causal attention of q [B, H, S, D] (S * H / KVH <= 16, D <= 64) over cache positions 0 .. pos+S-1: out
 * [B, S, H, D], the values of pai_sdpa_fwd with causal = 1, pos_offset = pos and the filled cache prefix. */
pai_status pai_sdpa_decode(pai_ctx* ctx, const pai_tensor* q, const pai_tensor* k_cache, const pai_tensor* v_cache,
                           const pai_tensor* pos, float scale, pai_tensor* out);
/* Decode-step products of one activation x [..., k] (at most 32 rows, contiguous rows) with up to four weights
 * W_i [n_i, k] (Linear.cs:10-43: y = x·Wᵀ), in one pass over the weights. With norm_weight (a [k] tensor, else NULL)
 * x is first normalised as pai_rmsnorm(x, norm_weight, eps) would (same values, bit for bit):
 *   mode 0: out [..., Σ n_i] = the products side by side (the attention's q, k and v projections);
 *   mode 1: out [..., n_0] = residual + x·W_0ᵀ (a Linear followed by TransformerBlock's residual Add, Modules.cs:222-246);
 *   mode 2: out [..., n_0] = SiLU(x·W_0ᵀ) ⊙ (x·W_1ᵀ) (SwiGluFeedForward's gate and up, Modules.cs:84-109).
 * The values are those of the separate MatMul / Add / SiluMul calls up to the summation order of the dot products. */
pai_status pai_linear_fused(pai_ctx* ctx, const pai_tensor* x, const pai_tensor* norm_weight, float eps,
                            const pai_tensor* weights, int32_t n_weights, int32_t mode, const pai_tensor* residual,
                            pai_tensor* out);
/* Captures every op issued on the context between begin and end into one CUDA graph; no host upload or
 * synchronising call may come in between. The device memory the captured ops use stays reserved for the graph
 * until pai_graph_destroy, so tensors created during the capture hold each replay's results. */
pai_status pai_graph_begin(pai_ctx* ctx);
pai_status pai_graph_end(pai_ctx* ctx, pai_graph** graph);
pai_status pai_graph_launch(pai_ctx* ctx, pai_graph* graph);
pai_status pai_graph_destroy(pai_ctx* ctx, pai_graph* graph);

/* ==== Data parallel (one process per GPU; no counterpart in the single-device reference) ==== */
pai_status pai_nccl_unique_id(uint8_t id_out[128]);
pai_status pai_nccl_init(pai_ctx* ctx, const uint8_t id[128], int32_t rank, int32_t world_size, int32_t timeout_ms);
/* Sum-all-reduce a bucket of contiguous F32 tensors in place on the communication stream, ordered after all
 * work queued so far on the compute stream; later compute-stream work that touches the bucket waits for it. */
pai_status pai_allreduce_bucket(pai_ctx* ctx, const pai_tensor* tensors, int32_t n_tensors);
/* ZeRO-1 exchanges (sharded AdamW state; the reference's AdamW, Optimizers.cs:81-123, keeps every moment on every
 * device). Rank r owns elements [r·n/W, (r+1)·n/W) of each tensor; n must divide by the world size W. reduce_scatter
 * sums every rank's tensor and leaves the sum of this rank's shard in place (other elements are unspecified
 * afterwards); allgather copies each rank's shard into every rank's tensor. Ordered like pai_allreduce_bucket and
 * completed by pai_allreduce_wait. */
pai_status pai_reduce_scatter_bucket(pai_ctx* ctx, const pai_tensor* tensors, int32_t n_tensors);
pai_status pai_allgather_bucket(pai_ctx* ctx, const pai_tensor* tensors, int32_t n_tensors);
/* Waits on the host, under the communicator's timeout, for every all-reduce issued so far, then orders the compute
 * stream after them. A failed or unfinished exchange (a peer left) aborts the communicator and returns PAI_ERR_NCCL or
 * PAI_ERR_TIMEOUT. Extends the step of ProjectAI.Training/Training.cs:87-113 with the cross-rank gradient sum. */
pai_status pai_allreduce_wait(pai_ctx* ctx);
pai_status pai_nccl_abort(pai_ctx* ctx);
/* Exposed exchange time since the last call: summed device milliseconds by which the last all-reduce of each step
 * ended after the step's backward (0 for a step whose exchange was hidden), and the number of steps counted. */
pai_status pai_dp_stats(pai_ctx* ctx, double* exposed_ms, int64_t* steps);

/* ==== Checkpoints: the PAICKPT2 format of ProjectAI.Formats/Checkpoint.cs:11-110, byte for byte ==== */
/* Checkpoint.Save (Checkpoint.cs:23-57): writes `path` with `step`, the metadata bytes and n_tensors F32 tensors, the
 * i-th named by the i-th NUL-terminated string packed into names[0, names_len). The tensors are copied once into a
 * device snapshot on the compute stream; a writer thread then streams the snapshot to the file through pinned host
 * chunks on a copy stream of its own, so the call returns while the file is written and later ops may change the
 * tensors. pai_ckpt_wait joins the writer and returns its status (PAI_ERR_IO on a failed write); a second save, or
 * destroying the context, waits for the first. Without device memory for the snapshot the save streams from the
 * tensors themselves and returns once the file is written. PAI_ERR_UNSUPPORTED for a tensor over 2^31 elements
 * (Checkpoint.cs:41-42), PAI_ERR_IO when the file cannot be created. */
pai_status pai_ckpt_save(pai_ctx* ctx, const char* path, int32_t step, const char* metadata, int64_t meta_len,
                         const char* names, int64_t names_len, const pai_tensor* tensors, int32_t n_tensors);
pai_status pai_ckpt_wait(pai_ctx* ctx);
/* Checkpoint.Load / ReadMetadata (Checkpoint.cs:59-139): reads the header (step, metadata length) and, unless
 * header_only, every tensor onto the device (F32, allocated in the current scope; the file is read chunk by chunk
 * while the previous chunk crosses to the device). The checks and messages are the reference's: PAI_ERR_INVALID_DATA
 * for a bad magic, metadata length, tensor count, name length, rank, dimension or payload length, or a truncated
 * file; PAI_ERR_IO when the file cannot be opened. pai_ckpt_meta copies the metadata bytes; pai_ckpt_tensor returns
 * the index-th tensor and its name (name_len bytes, no terminator); pai_ckpt_close forgets them (the tensors stay
 * allocated in their scope). */
pai_status pai_ckpt_load(pai_ctx* ctx, const char* path, int32_t header_only, int32_t* step, int64_t* meta_len,
                         int32_t* n_tensors);
pai_status pai_ckpt_meta(pai_ctx* ctx, char* buf, int64_t cap);
pai_status pai_ckpt_tensor(pai_ctx* ctx, int32_t index, char* name, int64_t name_cap, int64_t* name_len, pai_tensor* out);
pai_status pai_ckpt_close(pai_ctx* ctx);

/* ==== Packed token datasets (ProjectAI.Training/PackedBinDataset.cs:43-117, Training.cs:122-141) ==== */
/* PackedBinDataset.Open after its manifest is read: maps the shard, block_count blocks of seq_len + 1 little-endian ids
 * of elem_bytes each (2 = "u16", 4 = "u32"). PAI_ERR_INVALID_DATA for another width, seq_len < 1, block_count < 1 or a
 * shard shorter than the blocks need (PackedBinDataset.cs:62-83); PAI_ERR_IO when the shard cannot be opened. One
 * dataset per context; opening another replaces it. */
pai_status pai_dataset_open(pai_ctx* ctx, const char* bin_path, int32_t elem_bytes, int32_t seq_len, int64_t block_count);
/* NextBatch for the given block indices: inputs and targets [count, seq_len] F32 ids on the device (ids[:, :-1] and
 * ids[:, 1:] of each block), allocated in the current scope. The blocks are gathered from the mapping into pinned
 * memory at the shard's width, uploaded with one copy and widened on the device. PAI_ERR_OUT_OF_RANGE for an index
 * outside [0, block_count) (GetSequence, PackedBinDataset.cs:98-99) or a u32 id above int32 (its checked cast). */
pai_status pai_dataset_batch(pai_ctx* ctx, const int64_t* indices, int32_t count, pai_tensor* inputs, pai_tensor* targets);
pai_status pai_dataset_close(pai_ctx* ctx);

/* ==== Diagnostics (no counterpart in the reference; used by the benchmark and tests) ==== */
/* Reads and clears the device flag that bounded waits inside kernels set on a timeout (PAI_ERR_TIMEOUT if set). */
pai_status pai_check_device_error(pai_ctx* ctx, int32_t* code);
/* Device time between two points of the compute stream, from CUDA events recorded on that stream. stop blocks. */
pai_status pai_timer_start(pai_ctx* ctx);
pai_status pai_timer_stop(pai_ctx* ctx, float* ms);
/* Number of kernels this context has launched so far. */
pai_status pai_launch_count(pai_ctx* ctx, int64_t* n);
/* Per-kernel-family event timing ("gemm" = the tcgen05 GEMM kernel, "attn_fwd", "attn_bwd"). Enabling clears
 * previous samples. stats returns launches, summed device milliseconds and summed algorithmic work (flops). */
pai_status pai_kernel_timing(pai_ctx* ctx, int32_t enable);
pai_status pai_kernel_stats(pai_ctx* ctx, const char* family, int64_t* launches, double* total_ms, double* work);

#ifdef __cplusplus
}
#endif

#endif /* PROJECTAI_CUDA_H */
