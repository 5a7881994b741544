// C++ host runtime for the B200 backend: a restatement of the reference's C# host layer that sits above the
// IComputeBackend seam — Tensor views (ProjectAI.Core/Tensor.cs), the autograd facade and tape (Autograd.cs,
// GradNode.cs, GradMode.cs), PcgRng / Init (Rng.cs, Init.cs), Module (Module.cs), the Llama modules
// (ProjectAI.Models/*.cs), AdamW (Optimizers.cs), the trainer (ProjectAI.Training/Training.cs) and KV-cache decode
// (Inference.cs, Sampling.cs). It drives a backend library through the C ABI of include/projectai_cuda.h, bound at
// run time by path and symbol prefix (the CUDA library's prefix is "pai_").
//
// Where the backend offers the fused extensions (SDPA, RMSNorm backward, SiLU·Mul, fused cross-entropy, AdamW
// step), the autograd records one node per fused op; otherwise it records the reference's composed op chain.
#pragma once

#include <cstdint>
#include <utility>
#include <functional>
#include <map>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_set>
#include <vector>

#include "projectai_cuda.h"

namespace paihost {

// ---------------------------------------------------------------- errors (the .NET exception classes)
struct BackendError : std::runtime_error { using std::runtime_error::runtime_error; };
struct ArgumentError : BackendError { using BackendError::BackendError; };
struct OutOfRangeError : ArgumentError { using ArgumentError::ArgumentError; };
struct InvalidOperationError : BackendError { using BackendError::BackendError; };
struct OutOfMemoryError : BackendError { using BackendError::BackendError; };
struct DeviceTimeoutError : BackendError { using BackendError::BackendError; };
struct FileIOError : BackendError { using BackendError::BackendError; };       // IOException
struct InvalidDataError : BackendError { using BackendError::BackendError; };  // InvalidDataException

using Dims = std::vector<int>;
int64_t numel(const Dims& d);
std::string dims_str(const Dims& d);
std::vector<int64_t> contiguous_strides(const Dims& d);
Dims broadcast_dims(const Dims& a, const Dims& b);  // Shape.BroadcastWith (Shape.cs:86-113)

class NativeBackend;
struct GradNode;

// One backend allocation. Freed when its last view dies (unless a scope already freed it), when its scope ends
// (unless kept alive), or by Release.
struct Storage {
  NativeBackend* backend = nullptr;
  void* base = nullptr;
  int64_t count = 0;
  int scope = -1;       // index of the owning open scope, or -1
  bool freed = false;
  // Host copy of data uploaded by FromHost (ids, targets, constants): ToHost of an unmodified upload is served from it.
  std::shared_ptr<std::vector<float>> shadow;
  ~Storage();
};

struct TensorImpl;
using Tensor = std::shared_ptr<TensorImpl>;

// Tensor.cs:17-265: a view (shape, element strides, element offset) over shared storage, plus autograd metadata.
struct TensorImpl {
  Dims shape;
  std::vector<int64_t> strides;
  int64_t offset = 0;
  std::shared_ptr<Storage> storage;
  bool requires_grad = false;
  Tensor grad;
  std::shared_ptr<GradNode> grad_fn;
  NativeBackend* backend = nullptr;  // set by the autograd facade (Tensor.Backend)
  std::optional<float> known;        // value of a one-element tensor the host already knows (no read-back needed)

  int rank() const { return (int)shape.size(); }
  int64_t numel() const { return paihost::numel(shape); }
  bool is_contiguous() const;
  pai_tensor desc() const;
  // views (metadata only; detached: requires_grad = false)
  Tensor reshape(const Dims& d) const;
  Tensor transpose(int a0, int a1) const;
  Tensor permute(const std::vector<int>& p) const;
  Tensor slice(int axis, int start, int length) const;
  Tensor broadcast_to(const Dims& target) const;
  void backward();  // Tensor.Backward (Tensor.cs:213-252)
  // The same walk seeded with a given gradient of this tensor's shape instead of the scalar 1.
  void backward(const Tensor& seed);
};

Tensor make_view(const TensorImpl& t, Dims shape, std::vector<int64_t> strides, int64_t offset);

// ---------------------------------------------------------------- backend (the IComputeBackend seam)
struct OpTable;

class NativeBackend {
 public:
  NativeBackend(const std::string& library_path, const std::string& prefix, int device);
  ~NativeBackend();
  NativeBackend(const NativeBackend&) = delete;
  NativeBackend& operator=(const NativeBackend&) = delete;

  std::string name() const;
  bool has_fused() const;   // SDPA, RMSNorm backward, SiLU·Mul, fused CE, AdamW step
  bool use_fused = true;    // callers may turn the extensions off to run the reference's composed chains
  bool has_dp() const;

  // allocation & transfer (IComputeBackend.cs:14-18)
  Tensor allocate(const Dims& shape);
  Tensor from_host(const float* data, int64_t count, const Dims& shape);
  void to_host(const Tensor& t, float* dst, int64_t count);
  void copy(const Tensor& src, const Tensor& dst);
  // elementwise
  Tensor add(const Tensor& a, const Tensor& b);
  Tensor sub(const Tensor& a, const Tensor& b);
  Tensor mul(const Tensor& a, const Tensor& b);
  Tensor div(const Tensor& a, const Tensor& b);
  Tensor add_scalar(const Tensor& a, float s);
  Tensor mul_scalar(const Tensor& a, float s);
  Tensor sqrt(const Tensor& x);
  Tensor sigmoid(const Tensor& x);
  Tensor matmul(const Tensor& a, const Tensor& b, bool transpose_b = false);
  Tensor sum(const Tensor& x, int axis, bool keep = false);
  Tensor mean(const Tensor& x, int axis, bool keep = false);
  Tensor max(const Tensor& x, int axis, bool keep = false);
  Tensor softmax(const Tensor& x, int axis);
  Tensor rms_norm(const Tensor& x, const Tensor& w, float eps);
  Tensor silu(const Tensor& x);
  Tensor rotary(const Tensor& x, const Tensor& cos, const Tensor& sin);
  Tensor gather(const Tensor& table, const std::vector<int>& ids);
  Tensor scatter_add_rows(const Tensor& rows, const std::vector<int>& ids, int row_count);
  Tensor cross_entropy(const Tensor& logits, const std::vector<int>& targets, int ignore);
  Tensor cross_entropy_grad(const Tensor& logits, const std::vector<int>& targets, int ignore);
  Tensor cat(const Tensor& a, const Tensor& b, int axis);
  // fused extensions
  std::pair<Tensor, Tensor> sdpa_fwd(const Tensor& q, const Tensor& k, const Tensor& v, float scale, bool causal, int pos);
  std::vector<Tensor> sdpa_bwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse,
                               const Tensor& dout, float scale, bool causal, int pos);
  std::pair<Tensor, Tensor> rms_norm_bwd(const Tensor& x, const Tensor& w, const Tensor& g, float eps);
  Tensor silu_mul(const Tensor& gate, const Tensor& up);
  std::pair<Tensor, Tensor> silu_mul_bwd(const Tensor& gate, const Tensor& up, const Tensor& g);
  std::pair<Tensor, Tensor> cross_entropy_fused(const Tensor& logits, const std::vector<int>& targets, int ignore, float scale);
  void adamw_step(const Tensor& p, const Tensor& g, const Tensor& m, const Tensor& v, float lr, float b1, float b2,
                  float eps, float wd, int t, float grad_scale);
  // scopes (IComputeBackend.cs:69-95)
  void begin_scope();
  void end_scope();
  void keep_alive(const Tensor& t);
  void release(const Tensor& t);
  void sync();
  void memory_stats(int64_t* in_use, int64_t* peak, int64_t* reserved);
  void reset_peak();
  // data parallel
  void nccl_unique_id(uint8_t out[128]);
  void nccl_init(const uint8_t id[128], int rank, int world, int timeout_ms);
  void allreduce(const std::vector<Tensor>& grads);
  void allreduce_wait();
  // Aborts the communicator (no wait for peers): a rank leaving a job, or after a failed exchange.
  void nccl_abort();
  // ZeRO-1 exchanges: in-place NCCL reduce-scatter / all-gather of contiguous tensors whose element count divides by
  // the world size (rank r's shard is elements [r·n/W, (r+1)·n/W)); completed by allreduce_wait.
  void reduce_scatter(const std::vector<Tensor>& grads);
  void allgather(const std::vector<Tensor>& params);
  // Exposed all-reduce device time (ms summed over steps) and the step count since the last call.
  std::pair<double, int64_t> dp_stats();
  int dp_world = 1, dp_rank = 0;
  // decode steps with device-side ids and position, replayed as CUDA graphs (CUDA library only)
  bool has_graphs() const;
  void write(const Tensor& dst, const float* data, int64_t count);
  Tensor gather_dev(const Tensor& table, const Tensor& ids);
  Tensor rotary_at(const Tensor& x, const Tensor& cos_table, const Tensor& sin_table, const Tensor& pos);
  void kv_append(const Tensor& k, const Tensor& v, const Tensor& k_cache, const Tensor& v_cache, const Tensor& pos);
  Tensor sdpa_decode(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache, const Tensor& pos, float scale);
  // fused decode-step ops: x·Wᵀ over several weights with a store / residual / SiLU·mul epilogue, and RoPE + KV append
  bool has_decode_fusions() const;
  // index of each row's largest entry (ArgMax's rules, Sampling.cs:15-31) as a [rows] float tensor; optional op
  bool has_argmax_rows() const;
  Tensor argmax_rows(const Tensor& x);
  // PAICKPT2 checkpoints (Checkpoint.cs:23-139): save returns once the tensors are snapshotted on the device; the file
  // is written in the background until wait_checkpoint. load returns the tensors in the current scope.
  void save_checkpoint(const std::string& path, int step, const std::vector<std::pair<std::string, Tensor>>& tensors,
                       const std::string& metadata);
  void wait_checkpoint();
  struct LoadedCheckpoint {
    int step = 0;
    std::string metadata;
    std::vector<std::pair<std::string, Tensor>> tensors;
  };
  LoadedCheckpoint load_checkpoint(const std::string& path, bool header_only = false);
  // Packed token datasets (PackedBinDataset.cs): map a shard, then device [count, seq] F32 input/target ids per batch.
  void dataset_open(const std::string& bin_path, const std::string& dtype, int seq_len, int64_t block_count);
  std::pair<Tensor, Tensor> dataset_batch(const std::vector<int64_t>& indices);
  void dataset_close();
  Tensor linear_fused(const Tensor& x, const std::vector<Tensor>& weights, int mode, const Tensor& residual = nullptr,
                      const Tensor& norm_weight = nullptr, float eps = 0.0f);
  Tensor rope_append(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& cos_table, const Tensor& sin_table,
                     const Tensor& k_cache, const Tensor& v_cache, const Tensor& pos);
  Tensor attn_decode_step(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& cos_table, const Tensor& sin_table,
                          const Tensor& k_cache, const Tensor& v_cache, const Tensor& pos, float scale);
  void graph_begin();
  pai_graph* graph_end();
  void graph_launch(pai_graph* g);
  void graph_destroy(pai_graph* g);
  // diagnostics (CUDA library only)
  void timer_start();
  float timer_stop();
  int64_t launch_count();
  void kernel_timing(bool on);
  void kernel_stats(const std::string& family, int64_t* launches, double* ms, double* work);
  void check_device_error();

  // internals used by Storage
  void free_storage(Storage* s);
  pai_ctx* ctx() const { return ctx_; }

 private:
  friend struct Storage;
  Tensor wrap(const pai_tensor& d);
  void check(int status) const;
  Tensor unary(int which, const Tensor& x, float s = 0.0f);
  Tensor binary(int which, const Tensor& a, const Tensor& b);
  Tensor reduce(int which, const Tensor& x, int axis, bool keep);
  void invalidate_shadow(const Tensor& t);

  void* lib_ = nullptr;
  std::unique_ptr<OpTable> fn_;
  pai_ctx* ctx_ = nullptr;
  std::vector<std::unordered_set<Storage*>> scopes_;
  std::unordered_set<Storage*> live_;  // every Storage object still referring to this backend
};

// ---------------------------------------------------------------- autograd (GradMode.cs, GradNode.cs, Autograd.cs)
struct GradMode {
  static bool enabled();
  struct Guard {
    explicit Guard(bool disabled);
    ~Guard();
    bool previous;
  };
};

struct GradNode {
  std::string op;
  std::vector<Tensor> inputs;
  std::function<std::vector<Tensor>(const Tensor&)> backward;
};

class Autograd {
 public:
  explicit Autograd(NativeBackend* backend) : be(backend) {}
  NativeBackend* be;

  Tensor add(const Tensor& a, const Tensor& b);
  Tensor sub(const Tensor& a, const Tensor& b);
  Tensor mul(const Tensor& a, const Tensor& b);
  Tensor matmul(const Tensor& a, const Tensor& b, bool transpose_b = false);
  Tensor contiguous(const Tensor& x);
  Tensor sum_all(const Tensor& x);
  Tensor mean(const Tensor& x);
  Tensor checkpoint(const std::function<Tensor(const Tensor&)>& segment, const Tensor& input,
                    const std::vector<Tensor>& parameters, const std::function<void()>& on_grads_ready = nullptr);
  Tensor embedding(const Tensor& weight, const std::vector<int>& ids);
  Tensor cross_entropy(const Tensor& logits, const std::vector<int>& targets, int ignore);
  Tensor softmax(const Tensor& x, int axis);
  Tensor silu(const Tensor& x);
  Tensor rms_norm(const Tensor& x, const Tensor& w, float eps);
  Tensor rotary(const Tensor& x, const Tensor& cos, const Tensor& sin);
  // with the backward's −sin table supplied (no per-call negation)
  Tensor rotary(const Tensor& x, const Tensor& cos, const Tensor& sin, const Tensor& neg_sin);
  Tensor transpose(const Tensor& x, int a0, int a1);
  Tensor permute(const Tensor& x, const std::vector<int>& p);
  Tensor reshape(const Tensor& x, const Dims& d);
  Tensor slice(const Tensor& x, int axis, int start, int length);
  Tensor broadcast_to(const Tensor& x, const Dims& target);
  // fused extensions: one node each (composed fallbacks when the backend lacks them)
  Tensor silu_mul(const Tensor& gate, const Tensor& up);
  Tensor attention(const Tensor& q, const Tensor& k, const Tensor& v, float scale, int pos_offset);  // -> [B,S,H,D]

  float to_scalar(const Tensor& t);
  Tensor reduce_grad_to_shape(const Tensor& g, const Dims& target);

 private:
  Tensor record(const Tensor& y, const std::string& op, std::vector<Tensor> inputs,
                std::function<std::vector<Tensor>(const Tensor&)> backward);
  Tensor detach_leaf(const Tensor& x);
};

// ---------------------------------------------------------------- Rng / Init (Rng.cs, Init.cs)
class PcgRng {
 public:
  explicit PcgRng(uint64_t seed, uint64_t stream = 0xDA3E39CB94B95BDBull);
  uint32_t next_u32();
  float next_float();
  float next_gaussian();

 private:
  uint64_t state_, inc_;
  bool has_spare_ = false;
  float spare_ = 0.0f;
};

enum class InitKind { Zeros, Ones, Normal, Xavier, Kaiming };
struct Initializer {
  InitKind kind = InitKind::Normal;
  float a = 0.0f, b = 0.02f;  // Normal: mean, std; Xavier/Kaiming: gain
  void fill(const Tensor& target, NativeBackend& be, PcgRng& rng) const;
};

// ---------------------------------------------------------------- modules (Module.cs, ProjectAI.Models)
struct ModelConfig {
  int vocab_size = 256, embedding_dim = 128, layer_count = 2, head_count = 4, kv_head_count = 4, ffn_hidden = 344;
  int max_sequence_length = 4096;
  float rope_theta = 10000.0f, norm_eps = 1e-5f;
  int head_dim() const { return embedding_dim / head_count; }
  void validate() const;
};

struct ParameterContext {
  NativeBackend* backend;
  Autograd* ag;
  PcgRng* rng;
  bool skip_init = false;
  // Overrides every parameter's initializer (the configs that specify N(0, 0.02) weights for all matrices).
  std::optional<Initializer> override_init;
};

class KvCache;

struct ForwardContext {
  KvCache* cache = nullptr;
};

class Module {
 public:
  explicit Module(ParameterContext ctx) : ctx_(ctx) {}
  virtual ~Module() = default;
  std::vector<Tensor> parameters() const;
  std::vector<std::pair<std::string, Tensor>> named_parameters() const;

 protected:
  Tensor param(const std::string& name, const Dims& shape, Initializer init);
  template <class T>
  T* register_module(const std::string& name, std::unique_ptr<T> m) {
    T* raw = m.get();
    children_.emplace_back(name, std::move(m));
    return raw;
  }
  ParameterContext ctx_;
  Autograd& ag() const { return *ctx_.ag; }
  NativeBackend& be() const { return *ctx_.backend; }

 private:
  std::vector<std::pair<std::string, Tensor>> params_;
  std::vector<std::pair<std::string, std::unique_ptr<Module>>> children_;
};

class Linear : public Module {
 public:
  Linear(ParameterContext ctx, int in_dim, int out_dim, Initializer init);
  Tensor forward(const Tensor& x);
  Tensor weight;
  int in_dim, out_dim;
};

class RmsNorm : public Module {
 public:
  RmsNorm(ParameterContext ctx, int dim, float eps);
  Tensor forward(const Tensor& x);
  Tensor weight;
  float eps;
};

class RotaryEmbedding : public Module {
 public:
  RotaryEmbedding(ParameterContext ctx, int head_dim, float theta, int max_seq);
  Tensor apply_at_offset(const Tensor& x, int offset);
  // The same rotation of x [b, s, heads, dh] (positions on axis 1), the tables broadcast over the heads.
  Tensor apply_seq_major(const Tensor& x, int offset);
  Tensor cos, sin;
  Tensor neg_sin;  // −sin, the backward's table (RotaryEmbedding's backward, Autograd.cs:250-255), built once
  int max_seq;
};

class SwiGlu : public Module {
 public:
  SwiGlu(ParameterContext ctx, int dim, int hidden);
  Tensor forward(const Tensor& x);
  Linear *gate, *up, *down;
};

class Attention : public Module {
 public:
  Attention(ParameterContext ctx, const ModelConfig& cfg, int layer);
  Tensor forward(const Tensor& x, const ForwardContext& fctx);
  ModelConfig cfg;
  int layer;
  Linear *wq, *wk, *wv, *wo;
  RotaryEmbedding* rope;
  Tensor inv_sqrt_hd;

 private:
  Tensor causal_mask(int q_len, int k_len, int pos_offset);
};

class TransformerBlock : public Module {
 public:
  TransformerBlock(ParameterContext ctx, const ModelConfig& cfg, int layer);
  Tensor forward(const Tensor& x, const ForwardContext& fctx);
  RmsNorm *attn_norm, *ffn_norm;
  Attention* attn;
  SwiGlu* ffn;
};

class Embedding : public Module {
 public:
  Embedding(ParameterContext ctx, int vocab, int dim);
  Tensor forward(const Tensor& ids);
  Tensor weight;
  int vocab, dim;
};

class LlamaModel : public Module {
 public:
  LlamaModel(ParameterContext ctx, const ModelConfig& cfg);
  Tensor forward(const Tensor& ids, const ForwardContext& fctx = {});
  ModelConfig cfg;
  bool gradient_checkpointing = false;
  // Called after each checkpointed block's recompute has produced that block's parameter gradients.
  std::function<void(int block)> on_block_grads_ready;
  Embedding* embedding;
  std::vector<TransformerBlock*> blocks;
  RmsNorm* final_norm;
};

// Modules.cs:290-370: per-layer K/V of the positions seen so far. The reference grows each layer with Cat (the
// first append round-trips through the host); here each layer's storage [batch, kv_heads, max_seq, head_dim] is
// allocated on the device at the first append and later appends copy into it in place, so a decode step moves
// only the new positions. Append returns views of the filled prefix with the same values Cat would produce.
class KvCache {
 public:
  KvCache(NativeBackend* be, const ModelConfig& cfg, int max_batch, int max_seq);
  int length(int layer) const;
  std::pair<Tensor, Tensor> append(int layer, const Tensor& k, const Tensor& v);
  void reset();
  int max_batch, max_seq;
  // the whole per-layer storage (null before the first append) and, for appends written on the device
  // (NativeBackend::kv_append), the host-side length bookkeeping
  Tensor key_store(int layer) const { return key_store_.at((size_t)layer); }
  Tensor value_store(int layer) const { return value_store_.at((size_t)layer); }
  void advance(int positions);

 private:
  NativeBackend* be_;
  std::vector<Tensor> key_store_, value_store_;
  std::vector<int> lengths_;
};

std::vector<int> ids_from_tensor(NativeBackend& be, const Tensor& t);  // Embedding.ToIds / Loss.ToIds
Tensor cross_entropy_loss(Autograd& ag, const Tensor& logits, const Tensor& targets, int ignore = -100);  // Loss.cs

// ---------------------------------------------------------------- samplers (Sampling.cs)
int argmax(const float* logits, int n);
class TopKTopPSampler {
 public:
  TopKTopPSampler(uint64_t seed, float temperature, int top_k, float top_p) : rng(seed), temperature(temperature), top_k(top_k), top_p(top_p) {}
  int sample(const float* logits, int n);
  // Samples `batch` rows of `n` logits in row order (the RNG advances row by row exactly as repeated sample() calls);
  // each row's distribution is prepared on its own thread.
  void sample_rows(const float* rows, int batch, int n, int* out);
  // One row's distribution: `direct` >= 0 when the row falls back to argmax (no RNG draw), else the kept prefix of
  // the descending-probability order.
  struct Prepared {
    int direct = -1;
    int keep = 0;
    std::vector<int> order;
    std::vector<float> probs;
  };
  void prepare(const float* logits, int n, Prepared& p) const;
  int draw(const Prepared& p);
  PcgRng rng;
  float temperature;
  int top_k;
  float top_p;

 private:
  std::vector<Prepared> rows_;  // per-row buffers kept across sample_rows calls (a decode step reuses their storage)
};

// ---------------------------------------------------------------- optimizer (Optimizers.cs)
class AdamW {
 public:
  AdamW(std::vector<Tensor> params, NativeBackend* be, float lr = 1e-3f, float b1 = 0.9f, float b2 = 0.999f,
        float eps = 1e-8f, float wd = 0.01f);
  void step();
  void zero_grad();
  std::function<float(int)> schedule;
  float lr, b1, b2, eps, wd;
  int step_count = 0;
  float grad_scale = 1.0f;  // 1/world for a data-parallel sum
  // ZeRO-1: with shard_world > 1 this rank updates only its shard of each parameter whose element count divides by
  // shard_world (elements [r·n/W, (r+1)·n/W) of the flattened tensor) and keeps moments for that shard alone; the
  // others are updated whole. The caller exchanges the shards (reduce-scatter before, all-gather after).
  int shard_rank = 0, shard_world = 1;
  bool sharded(const Tensor& p) const { return shard_world > 1 && p->numel() % shard_world == 0; }
  struct State { Tensor m, v; int t = 0; };
  std::map<TensorImpl*, State> state;

 private:
  std::vector<Tensor> params_;
  NativeBackend* be_;
};

// ---------------------------------------------------------------- training (Training.cs)
struct TrainingConfig {
  int batch_size = 8, sequence_length = 512;
  float learning_rate = 3e-4f, weight_decay = 0.01f;
  int max_steps = 1000, grad_accum = 1;
  bool gradient_checkpointing = false;
  int warmup_steps = 100;
  uint64_t seed = 0;
  // Trainer::train writes "<checkpoint_directory>/step-<n>.ckpt" every checkpoint_every_steps steps (0: only the
  // final one) and after the last step; an empty directory writes none (TrainingConfig, Training.cs:8-26).
  int checkpoint_every_steps = 0;
  std::string checkpoint_directory = "checkpoints";
};

// A source of training sequences for Trainer::train (IDataset, Training.cs:29-33): count() sequences, and NextBatch's
// [rows, seq] input and target id tensors for the drawn row indices (inputs ids[:, :seq], targets ids[:, 1:seq+1]).
struct SequenceSource {
  virtual ~SequenceSource() = default;
  virtual int64_t count() const = 0;
  virtual std::pair<Tensor, Tensor> batch(NativeBackend* be, const std::vector<int64_t>& rows, int seq) = 0;
};

// Sequences held on the host (int token ids), uploaded per batch as NextBatch does (Training.cs:122-141), with its
// length check.
struct HostSequences : SequenceSource {
  std::vector<std::vector<int32_t>> seqs;
  int64_t count() const override { return (int64_t)seqs.size(); }
  std::pair<Tensor, Tensor> batch(NativeBackend* be, const std::vector<int64_t>& rows, int seq) override;
};

// The packed dataset the backend has open (NativeBackend::dataset_open, PackedBinDataset.cs): blocks gathered at
// their on-disk width and widened to F32 ids on the device.
struct PackedSequences : SequenceSource {
  int64_t blocks = 0;
  int64_t count() const override { return blocks; }
  std::pair<Tensor, Tensor> batch(NativeBackend* be, const std::vector<int64_t>& rows, int seq) override;
};

// Checkpointing.ApplyWeights (Checkpointing.cs:128-137): copies each saved weight into the model parameter of the same
// name, raising InvalidDataError for a missing parameter or a shape mismatch.
void apply_weights(NativeBackend* be, LlamaModel* model, const std::vector<std::pair<std::string, Tensor>>& items);

// Per-step mean losses and the final step of a run (TrainingReport, Training.cs:36-41).
struct TrainingReport {
  std::vector<float> step_losses;
  int final_step = 0;
};

std::function<float(int)> warmup_cosine(const TrainingConfig& cfg);

// One training step in the reference trainer's order (Training.cs:87-113): ZeroGrad, per micro-batch scope
// {forward, loss, ToHost(loss), backward, KeepAlive(grads)}, optimizer step. Batches come from the caller.
class Trainer {
 public:
  Trainer(NativeBackend* be, LlamaModel* model, const TrainingConfig& cfg, float beta1 = 0.9f, float beta2 = 0.999f);
  // inputs/targets: micro-batches of [batch, seq] token ids (row-major) as floats, one pair per micro step.
  float step(const std::vector<std::vector<float>>& inputs, const std::vector<std::vector<float>>& targets);
  // The same step on batches already uploaded to the device ([batch, seq] id tensors from FromHost).
  float step_tensors(const std::vector<Tensor>& inputs, const std::vector<Tensor>& targets);
  // Checkpointing.SaveModel's state (Checkpointing.cs:103-115: each parameter by name, then its AdamW moments as
  // "opt.m::name" / "opt.v::name") written as PAICKPT2 with `step`; the file is finished by wait_checkpoint (or the
  // next save). restore (Training.cs:156-162 with Checkpointing.ApplyWeights / ApplyOptimizer) copies the weights and
  // moments back, sets the optimizer's step count and returns the saved step.
  //
  // Under ZeRO-1 the moments of sharded parameters live one shard per rank, so save_checkpoint is collective: every
  // rank calls it, the shards are all-gathered into full-size moments (the file is the same as a replicated run's),
  // and a rank that passes an empty path joins the gather without writing. restore reads the full file on each rank
  // and keeps this rank's shard of every sharded moment.
  void save_checkpoint(const std::string& path, int step, const std::string& metadata = "");
  void wait_checkpoint();
  int restore(const std::string& path);
  // The state save_checkpoint writes, in its order, with full-size moments (collective under ZeRO-1; the tensors
  // belong to the caller's scope), and the part of restore that applies such a state and step count.
  std::vector<std::pair<std::string, Tensor>> state_items();
  void apply_state(const std::vector<std::pair<std::string, Tensor>>& items, int step);
  // Trainer.Train (Training.cs:59-120): max_steps steps of grad_accum micro-batches, each drawn by NextBatch's rule
  // (row = PcgRng(seed).NextUInt32() % count per batch row), the warmup+cosine schedule, a checkpoint every
  // checkpoint_every_steps steps and after the last one; on_step(step, loss) after each step. Returns once the last
  // checkpoint file is complete. Under data parallelism rank r draws from PCG stream (default + r) of the same seed
  // (rank 0: the reference's sequence), and rank 0 writes the files (every rank joins the gather under ZeRO-1).
  TrainingReport train(SequenceSource& data, const std::function<void(int, float)>& on_step = nullptr);
  LlamaModel* model;
  TrainingConfig cfg;
  std::unique_ptr<AdamW> optimizer;
  Autograd ag;
  // Data parallel: the number of ranks and the bucket exchange. Default: the backend's NCCL communicator
  // (world = backend.dp_world); callers may substitute another sum-all-reduce (e.g. a CPU collective in tests).
  int world = 0;  // 0: take the backend's dp_world
  int rank = -1;  // -1: take the backend's dp_rank
  std::function<void(const std::vector<Tensor>&)> allreduce;
  std::function<void()> allreduce_wait;
  // ZeRO-1 (optimizer state sharded over the ranks): gradients of shardable parameters are reduce-scattered instead
  // of all-reduced, AdamW updates this rank's shard, and the parameters are all-gathered after the update. The
  // exchanges default to the backend's NCCL communicator; tests substitute CPU collectives.
  bool zero1 = false;
  std::function<void(const std::vector<Tensor>&)> reduce_scatter;
  std::function<void(const std::vector<Tensor>&)> allgather;

 private:
  // Sets the optimizer's shard rank and world from world / rank / zero1 (the backend's when unset); returns the world.
  int configure_shards();
  NativeBackend* be_;
  std::vector<Tensor> params_;
  std::vector<std::vector<Tensor>> block_params_;
  std::vector<Tensor> tail_params_;
};

// Inference.cs:23-64 with a sampler: prefill, then one token per step through the KV cache.
// Decode steps of one lockstep batch (one new position per sequence) replayed as a CUDA graph: the ops of
// LlamaModel::forward with the KV cache for that shape (Modules.cs:142-204, 222-288), with the token ids and the position
// read from device tensors so the step captured once serves every later position. The first step runs eagerly (it warms
// the allocator), the second is captured and launched, later ones only launch. The cache must already hold the
// prompt (a prefill through LlamaModel::forward).
class GraphDecoder {
 public:
  GraphDecoder(NativeBackend* be, LlamaModel* model, KvCache* cache, int batch);
  ~GraphDecoder();
  // Runs one step for `ids` (one per sequence) at the cache's current length; returns logits [batch, 1, vocab], a
  // device tensor the next step overwrites.
  Tensor step(const std::vector<int>& ids);
  bool captured() const { return graph_ != nullptr; }
  bool fused = true;  // use the fused decode ops when the backend has them (false: one backend op per model op)

 private:
  Tensor body();
  Tensor body_fused();
  NativeBackend* be_;
  LlamaModel* model_;
  KvCache* cache_;
  int batch_;
  Tensor ids_, pos_, logits_;
  pai_graph* graph_ = nullptr;
  int steps_ = 0;
};

struct GenerateResult {
  std::vector<int> tokens;
  double prefill_seconds = 0, decode_seconds = 0;
  bool graph = false;  // the decode steps ran as a replayed CUDA graph
};
GenerateResult generate(NativeBackend* be, LlamaModel* model, const std::vector<int>& prompt, int max_tokens,
                        TopKTopPSampler* sampler, int batch = 1);

}  // namespace paihost
