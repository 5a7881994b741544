// Tensor views (ProjectAI.Core/Tensor.cs, Shape.cs), Tensor.Backward (Tensor.cs:213-261) and the run-time binding of a
// backend library's C ABI (the P/Invoke layer of a ProjectAI.Backends.Cuda project, restated in C++).
#include <dlfcn.h>

#include <algorithm>
#include <cstring>
#include <unordered_map>

#include "runtime.h"

namespace paihost {

int64_t numel(const Dims& d) {
  int64_t n = 1;
  for (int x : d) n *= x;
  return n;
}

std::string dims_str(const Dims& d) {
  std::string s = "[";
  for (size_t i = 0; i < d.size(); i++) {
    if (i) s += ", ";
    s += std::to_string(d[i]);
  }
  return s + "]";
}

std::vector<int64_t> contiguous_strides(const Dims& d) {
  std::vector<int64_t> s(d.size());
  int64_t acc = 1;
  for (int i = (int)d.size() - 1; i >= 0; i--) {
    s[(size_t)i] = acc;
    acc *= d[(size_t)i];
  }
  return s;
}

Dims broadcast_dims(const Dims& a, const Dims& b) {
  size_t n = std::max(a.size(), b.size());
  Dims r(n);
  for (size_t i = 0; i < n; i++) {
    int da = i < a.size() ? a[a.size() - 1 - i] : 1;
    int db = i < b.size() ? b[b.size() - 1 - i] : 1;
    if (da == db) r[n - 1 - i] = da;
    else if (da == 1) r[n - 1 - i] = db;
    else if (db == 1) r[n - 1 - i] = da;
    else throw ArgumentError("Shapes " + dims_str(a) + " and " + dims_str(b) + " are not broadcast-compatible.");
  }
  return r;
}

// ---------------------------------------------------------------- Storage
Storage::~Storage() {
  if (!backend) return;
  if (!freed) backend->free_storage(this);
  backend->live_.erase(this);
}

// ---------------------------------------------------------------- TensorImpl views (Tensor.cs:55-168)
bool TensorImpl::is_contiguous() const {
  int64_t acc = 1;
  for (int i = rank() - 1; i >= 0; i--) {
    if (shape[(size_t)i] == 1) continue;
    if (strides[(size_t)i] != acc) return false;
    acc *= shape[(size_t)i];
  }
  return true;
}

pai_tensor TensorImpl::desc() const {
  if (!storage || storage->freed)
    throw InvalidOperationError("tensor storage has been released (used after its scope ended?)");
  pai_tensor d;
  memset(&d, 0, sizeof d);
  d.base = storage->base;
  d.offset = offset;
  d.rank = rank();
  d.dtype = PAI_F32;
  if (rank() > PAI_MAX_RANK) throw ArgumentError("rank above 8 is not supported");
  for (int i = 0; i < rank(); i++) {
    d.dims[i] = shape[(size_t)i];
    d.strides[i] = strides[(size_t)i];
  }
  return d;
}

Tensor make_view(const TensorImpl& t, Dims shape, std::vector<int64_t> strides, int64_t offset) {
  auto r = std::make_shared<TensorImpl>();
  r->shape = std::move(shape);
  r->strides = std::move(strides);
  r->offset = offset;
  r->storage = t.storage;
  r->backend = t.backend;
  if (r->numel() == 1 && t.numel() == 1) r->known = t.known;
  return r;
}

Tensor TensorImpl::reshape(const Dims& d) const {
  if (!is_contiguous()) throw InvalidOperationError("Reshape requires a contiguous tensor; materialize it first.");
  for (int x : d)
    if (x < 0) throw OutOfRangeError("Dimensions must be non-negative.");
  if (paihost::numel(d) != numel())
    throw ArgumentError("Cannot reshape " + dims_str(shape) + " (" + std::to_string(numel()) + " elements) to " + dims_str(d) + ".");
  return make_view(*this, d, contiguous_strides(d), offset);
}

Tensor TensorImpl::transpose(int a0, int a1) const {
  if (a0 < 0 || a0 >= rank() || a1 < 0 || a1 >= rank()) throw OutOfRangeError("Transpose axis out of range.");
  Dims d = shape;
  auto s = strides;
  std::swap(d[(size_t)a0], d[(size_t)a1]);
  std::swap(s[(size_t)a0], s[(size_t)a1]);
  return make_view(*this, d, s, offset);
}

Tensor TensorImpl::permute(const std::vector<int>& p) const {
  if ((int)p.size() != rank()) throw ArgumentError("Permutation length does not match rank.");
  Dims d(p.size());
  std::vector<int64_t> s(p.size());
  std::vector<bool> seen(p.size(), false);
  for (size_t i = 0; i < p.size(); i++) {
    if (p[i] < 0 || p[i] >= rank() || seen[(size_t)p[i]]) throw ArgumentError("Permutation must be a rearrangement of 0..rank-1.");
    seen[(size_t)p[i]] = true;
    d[i] = shape[(size_t)p[i]];
    s[i] = strides[(size_t)p[i]];
  }
  return make_view(*this, d, s, offset);
}

Tensor TensorImpl::slice(int axis, int start, int length) const {
  if (axis < 0 || axis >= rank()) throw OutOfRangeError("Slice axis out of range.");
  int dim = shape[(size_t)axis];
  if (start < 0 || length < 0 || start + length > dim)
    throw OutOfRangeError("Slice [" + std::to_string(start) + ", " + std::to_string(start + length) + ") is out of range for axis " +
                          std::to_string(axis) + " (size " + std::to_string(dim) + ").");
  Dims d = shape;
  d[(size_t)axis] = length;
  return make_view(*this, d, strides, offset + (int64_t)start * strides[(size_t)axis]);
}

Tensor TensorImpl::broadcast_to(const Dims& target) const {
  if (shape.size() > target.size()) throw ArgumentError("Cannot broadcast " + dims_str(shape) + " to fewer dimensions " + dims_str(target) + ".");
  size_t lead = target.size() - shape.size();
  std::vector<int64_t> s(target.size());
  for (size_t i = 0; i < target.size(); i++) {
    if (i < lead) { s[i] = 0; continue; }
    int sd = shape[i - lead];
    if (sd == target[i]) s[i] = strides[i - lead];
    else if (sd == 1) s[i] = 0;
    else throw ArgumentError("Cannot broadcast " + dims_str(shape) + " to " + dims_str(target) + ".");
  }
  return make_view(*this, target, s, offset);
}

// Tensor.Backward (Tensor.cs:213-252): topological order, clear intermediate grads, seed ones, reverse walk with
// fan-out accumulation by Add.
void TensorImpl::backward() {
  if (!backend) throw InvalidOperationError("Backward requires a tensor produced by the Autograd facade (no graph/backend recorded).");
  if (numel() != 1)
    throw InvalidOperationError("Backward expects a scalar loss; this tensor has shape " + dims_str(shape) + ". Reduce to a scalar first.");
  Tensor seed = backend->add_scalar(backend->allocate(shape), 1.0f);
  seed->known = 1.0f;
  backward(seed);
}

void TensorImpl::backward(const Tensor& seed) {
  if (!backend) throw InvalidOperationError("Backward requires a tensor produced by the Autograd facade (no graph/backend recorded).");
  if (!seed || seed->shape != shape)
    throw ArgumentError("Backward seed must have the tensor's shape " + dims_str(shape) + ".");
  NativeBackend& be = *backend;
  std::vector<TensorImpl*> topo;
  std::vector<Tensor> keep;  // holds every node alive during the walk
  std::unordered_set<TensorImpl*> visited;
  // Iterative post-order DFS (the reference recurses; the order is the same).
  struct Frame { TensorImpl* t; size_t next; };
  std::vector<Frame> stack;
  visited.insert(this);
  stack.push_back({this, 0});
  while (!stack.empty()) {
    Frame& f = stack.back();
    if (f.t->grad_fn && f.next < f.t->grad_fn->inputs.size()) {
      const Tensor& in = f.t->grad_fn->inputs[f.next++];
      if (visited.insert(in.get()).second) {
        keep.push_back(in);
        stack.push_back({in.get(), 0});
      }
      continue;
    }
    topo.push_back(f.t);
    stack.pop_back();
  }
  for (TensorImpl* n : topo)
    if (n->grad_fn) n->grad.reset();
  grad = seed;
  for (int i = (int)topo.size() - 1; i >= 0; i--) {
    TensorImpl* node = topo[(size_t)i];
    if (!node->grad_fn || !node->grad) continue;
    std::shared_ptr<GradNode> fn = node->grad_fn;
    std::vector<Tensor> grads = fn->backward(node->grad);
    // An intermediate node's gradient is dead once its rule has run; drop it now instead of at scope end.
    node->grad.reset();
    for (size_t j = 0; j < fn->inputs.size(); j++) {
      const Tensor& input = fn->inputs[j];
      if (!input->requires_grad) continue;
      input->grad = input->grad ? be.add(input->grad, grads[j]) : grads[j];
    }
  }
}

// ---------------------------------------------------------------- NativeBackend: C ABI bound at run time
#define PAI_FN_LIST(X)                                                                                       \
  X(last_error, const char* (*)(void))                                                                       \
  X(ctx_create, int (*)(int, pai_ctx**))                                                                     \
  X(ctx_destroy, int (*)(pai_ctx*))                                                                          \
  X(sync, int (*)(pai_ctx*))                                                                                 \
  X(device_name, int (*)(pai_ctx*, char*, int32_t))                                                          \
  X(alloc, int (*)(pai_ctx*, int32_t, const int32_t*, int32_t, pai_tensor*))                                 \
  X(from_host, int (*)(pai_ctx*, const float*, int64_t, int32_t, const int32_t*, int32_t, pai_tensor*))      \
  X(to_host, int (*)(pai_ctx*, const pai_tensor*, float*, int64_t))                                          \
  X(copy, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*))                                           \
  X(scope_begin, int (*)(pai_ctx*))                                                                          \
  X(scope_end, int (*)(pai_ctx*))                                                                            \
  X(keep_alive, int (*)(pai_ctx*, const void*))                                                              \
  X(release, int (*)(pai_ctx*, const void*))                                                                 \
  X(memory_stats, int (*)(pai_ctx*, int64_t*, int64_t*, int64_t*))                                           \
  X(reset_peak, int (*)(pai_ctx*))                                                                           \
  X(add, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, pai_tensor*))                               \
  X(sub, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, pai_tensor*))                               \
  X(mul, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, pai_tensor*))                               \
  X(div, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, pai_tensor*))                               \
  X(add_scalar, int (*)(pai_ctx*, const pai_tensor*, float, pai_tensor*))                                    \
  X(mul_scalar, int (*)(pai_ctx*, const pai_tensor*, float, pai_tensor*))                                    \
  X(sqrt, int (*)(pai_ctx*, const pai_tensor*, pai_tensor*))                                                 \
  X(sigmoid, int (*)(pai_ctx*, const pai_tensor*, pai_tensor*))                                              \
  X(silu, int (*)(pai_ctx*, const pai_tensor*, pai_tensor*))                                                 \
  X(matmul, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, int32_t, pai_tensor*))                   \
  X(sum, int (*)(pai_ctx*, const pai_tensor*, int32_t, int32_t, pai_tensor*))                                \
  X(mean, int (*)(pai_ctx*, const pai_tensor*, int32_t, int32_t, pai_tensor*))                               \
  X(max, int (*)(pai_ctx*, const pai_tensor*, int32_t, int32_t, pai_tensor*))                                \
  X(softmax, int (*)(pai_ctx*, const pai_tensor*, int32_t, pai_tensor*))                                     \
  X(rmsnorm, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, float, pai_tensor*))                    \
  X(rotary, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, pai_tensor*))         \
  X(gather, int (*)(pai_ctx*, const pai_tensor*, const int32_t*, int64_t, pai_tensor*))                      \
  X(scatter_add_rows, int (*)(pai_ctx*, const pai_tensor*, const int32_t*, int64_t, int32_t, pai_tensor*))   \
  X(cross_entropy, int (*)(pai_ctx*, const pai_tensor*, const int32_t*, int64_t, int32_t, pai_tensor*))      \
  X(cross_entropy_grad, int (*)(pai_ctx*, const pai_tensor*, const int32_t*, int64_t, int32_t, pai_tensor*)) \
  X(cat, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, int32_t, pai_tensor*))

#define PAI_OPT_FN_LIST(X)                                                                                              \
  X(sdpa_fwd, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, float, int32_t, int32_t,        \
                      pai_tensor*, pai_tensor*))                                                                         \
  X(sdpa_bwd, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, const pai_tensor*,              \
                      const pai_tensor*, const pai_tensor*, float, int32_t, int32_t, pai_tensor*, pai_tensor*,           \
                      pai_tensor*))                                                                                      \
  X(rmsnorm_bwd, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, float, pai_tensor*,          \
                         pai_tensor*))                                                                                   \
  X(silu_mul_fwd, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, pai_tensor*))                                  \
  X(silu_mul_bwd, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, pai_tensor*, pai_tensor*))  \
  X(cross_entropy_fused, int (*)(pai_ctx*, const pai_tensor*, const int32_t*, int64_t, int32_t, float, pai_tensor*,      \
                                 pai_tensor*))                                                                           \
  X(adamw_step, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, const pai_tensor*, float,     \
                        float, float, float, float, int32_t, float))                                                     \
  X(finalize, int (*)(pai_ctx*, const void*))                                                                            \
  X(nccl_unique_id, int (*)(uint8_t*))                                                                                   \
  X(nccl_init, int (*)(pai_ctx*, const uint8_t*, int32_t, int32_t, int32_t))                                             \
  X(allreduce_bucket, int (*)(pai_ctx*, const pai_tensor*, int32_t))                                                     \
  X(allreduce_wait, int (*)(pai_ctx*))                                                                                  \
  X(dp_stats, int (*)(pai_ctx*, double*, int64_t*))                                                                      \
  X(nccl_abort, int (*)(pai_ctx*))                                                                                       \
  X(reduce_scatter_bucket, int (*)(pai_ctx*, const pai_tensor*, int32_t))                                                \
  X(allgather_bucket, int (*)(pai_ctx*, const pai_tensor*, int32_t))                                                     \
  X(timer_start, int (*)(pai_ctx*))                                                                                      \
  X(timer_stop, int (*)(pai_ctx*, float*))                                                                               \
  X(launch_count, int (*)(pai_ctx*, int64_t*))                                                                           \
  X(kernel_timing, int (*)(pai_ctx*, int32_t))                                                                           \
  X(kernel_stats, int (*)(pai_ctx*, const char*, int64_t*, double*, double*))                                            \
  X(check_device_error, int (*)(pai_ctx*, int32_t*))                                                                    \
  X(write, int (*)(pai_ctx*, const float*, int64_t, const pai_tensor*))                                                  \
  X(gather_dev, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, pai_tensor*))                                    \
  X(rotary_at, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, const pai_tensor*, pai_tensor*)) \
  X(kv_append, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, const pai_tensor*,             \
                       const pai_tensor*))                                                                               \
  X(sdpa_decode, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, const pai_tensor*, float,    \
                         pai_tensor*))                                                                                   \
  X(linear_fused, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, float, const pai_tensor*, int32_t, int32_t,   \
                          const pai_tensor*, pai_tensor*))                                                               \
  X(rope_append, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, const pai_tensor*,           \
                         const pai_tensor*, const pai_tensor*, const pai_tensor*, const pai_tensor*, pai_tensor*))       \
  X(attn_decode_step, int (*)(pai_ctx*, const pai_tensor*, const pai_tensor*, const pai_tensor*, const pai_tensor*,      \
                              const pai_tensor*, const pai_tensor*, const pai_tensor*, const pai_tensor*, float,         \
                              pai_tensor*))                                                                              \
  X(graph_begin, int (*)(pai_ctx*))                                                                                      \
  X(graph_end, int (*)(pai_ctx*, pai_graph**))                                                                           \
  X(graph_launch, int (*)(pai_ctx*, pai_graph*))                                                                         \
  X(graph_destroy, int (*)(pai_ctx*, pai_graph*))                                                                       \
  X(argmax_rows, int (*)(pai_ctx*, const pai_tensor*, pai_tensor*))                                                     \
  X(ckpt_save, int (*)(pai_ctx*, const char*, int32_t, const char*, int64_t, const char*, int64_t, const pai_tensor*,    \
                       int32_t))                                                                                         \
  X(ckpt_wait, int (*)(pai_ctx*))                                                                                        \
  X(ckpt_load, int (*)(pai_ctx*, const char*, int32_t, int32_t*, int64_t*, int32_t*))                                    \
  X(ckpt_meta, int (*)(pai_ctx*, char*, int64_t))                                                                        \
  X(ckpt_tensor, int (*)(pai_ctx*, int32_t, char*, int64_t, int64_t*, pai_tensor*))                                      \
  X(ckpt_close, int (*)(pai_ctx*))                                                                                       \
  X(dataset_open, int (*)(pai_ctx*, const char*, int32_t, int32_t, int64_t))                                             \
  X(dataset_batch, int (*)(pai_ctx*, const int64_t*, int32_t, pai_tensor*, pai_tensor*))                                 \
  X(dataset_close, int (*)(pai_ctx*))

template <class T>
using Fn = T;

struct OpTable {
#define DECL(name, type) Fn<type> name = nullptr;
  PAI_FN_LIST(DECL)
  PAI_OPT_FN_LIST(DECL)
#undef DECL
};

NativeBackend::NativeBackend(const std::string& path, const std::string& prefix, int device) : fn_(new OpTable()) {
  lib_ = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
  if (!lib_) throw BackendError(std::string("cannot load backend library: ") + dlerror());
#define LOAD(name, type)                                                                          \
  fn_->name = reinterpret_cast<type>(dlsym(lib_, (prefix + #name).c_str()));                      \
  if (!fn_->name) throw BackendError("backend library " + path + " lacks " + prefix + #name);
  PAI_FN_LIST(LOAD)
#undef LOAD
#define LOAD_OPT(name, type) fn_->name = reinterpret_cast<type>(dlsym(lib_, (prefix + #name).c_str()));
  PAI_OPT_FN_LIST(LOAD_OPT)
#undef LOAD_OPT
  check(fn_->ctx_create(device, &ctx_));
}

NativeBackend::~NativeBackend() {
  for (Storage* s : live_) {  // tensors that outlive the backend become dead handles
    s->backend = nullptr;
    s->freed = true;
  }
  if (ctx_) fn_->ctx_destroy(ctx_);
  // The library stays loaded: Storage objects that outlive this backend must not call into unmapped code.
}

void NativeBackend::check(int st) const {
  if (st == PAI_OK) return;
  std::string msg = fn_->last_error();
  switch (st) {
    case PAI_ERR_ARGUMENT: throw ArgumentError(msg);
    case PAI_ERR_OUT_OF_RANGE: throw OutOfRangeError(msg);
    case PAI_ERR_INVALID_OP: throw InvalidOperationError(msg);
    case PAI_ERR_OUT_OF_MEMORY: throw OutOfMemoryError(msg);
    case PAI_ERR_TIMEOUT: throw DeviceTimeoutError(msg);
    case PAI_ERR_IO: throw FileIOError(msg);
    case PAI_ERR_INVALID_DATA: throw InvalidDataError(msg);
    default: throw BackendError(msg);
  }
}

std::string NativeBackend::name() const {
  char buf[256] = {0};
  check(fn_->device_name(ctx_, buf, sizeof buf));
  return buf;
}

bool NativeBackend::has_fused() const {
  return fn_->sdpa_fwd && fn_->sdpa_bwd && fn_->rmsnorm_bwd && fn_->silu_mul_fwd && fn_->silu_mul_bwd &&
         fn_->cross_entropy_fused && fn_->adamw_step;
}

bool NativeBackend::has_dp() const { return fn_->nccl_init && fn_->allreduce_bucket && fn_->allreduce_wait; }

bool NativeBackend::has_graphs() const {
  return fn_->write && fn_->gather_dev && fn_->rotary_at && fn_->kv_append && fn_->sdpa_decode && fn_->graph_begin &&
         fn_->graph_end && fn_->graph_launch && fn_->graph_destroy;
}

bool NativeBackend::has_decode_fusions() const { return fn_->linear_fused && fn_->rope_append && fn_->attn_decode_step; }
bool NativeBackend::has_argmax_rows() const { return fn_->argmax_rows != nullptr; }

// ---------------------------------------------------------------- checkpoints and packed datasets (io.cu)
static void need_io(const void* fn, const char* what) {
  if (!fn) throw BackendError(std::string("backend has no ") + what + " (the CUDA backend provides it)");
}

void NativeBackend::save_checkpoint(const std::string& path, int step,
                                    const std::vector<std::pair<std::string, Tensor>>& tensors, const std::string& metadata) {
  need_io((void*)fn_->ckpt_save, "checkpoint I/O");
  std::string names;
  std::vector<pai_tensor> d;
  for (const auto& kv : tensors) {
    names += kv.first;
    names.push_back('\0');
    d.push_back(kv.second->desc());
  }
  check(fn_->ckpt_save(ctx_, path.c_str(), step, metadata.data(), (int64_t)metadata.size(), names.data(),
                       (int64_t)names.size(), d.data(), (int32_t)d.size()));
}

void NativeBackend::wait_checkpoint() {
  need_io((void*)fn_->ckpt_wait, "checkpoint I/O");
  check(fn_->ckpt_wait(ctx_));
}

NativeBackend::LoadedCheckpoint NativeBackend::load_checkpoint(const std::string& path, bool header_only) {
  need_io((void*)fn_->ckpt_load, "checkpoint I/O");
  LoadedCheckpoint r;
  int32_t count = 0;
  int64_t mlen = 0;
  check(fn_->ckpt_load(ctx_, path.c_str(), header_only ? 1 : 0, &r.step, &mlen, &count));
  r.metadata.resize((size_t)mlen);
  check(fn_->ckpt_meta(ctx_, mlen ? &r.metadata[0] : nullptr, mlen));
  for (int32_t i = 0; i < count; i++) {
    int64_t nlen = 0;
    check(fn_->ckpt_tensor(ctx_, i, nullptr, 0, &nlen, nullptr));
    std::string name((size_t)nlen, '\0');
    pai_tensor t;
    check(fn_->ckpt_tensor(ctx_, i, nlen ? &name[0] : nullptr, nlen, nullptr, &t));
    r.tensors.emplace_back(std::move(name), wrap(t));
  }
  check(fn_->ckpt_close(ctx_));
  return r;
}

void NativeBackend::dataset_open(const std::string& bin_path, const std::string& dtype, int seq_len, int64_t block_count) {
  need_io((void*)fn_->dataset_open, "packed datasets");
  const int width = dtype == "u16" ? 2 : dtype == "u32" ? 4 : 0;
  check(fn_->dataset_open(ctx_, bin_path.c_str(), width, seq_len, block_count));
}

std::pair<Tensor, Tensor> NativeBackend::dataset_batch(const std::vector<int64_t>& indices) {
  need_io((void*)fn_->dataset_batch, "packed datasets");
  pai_tensor in, tg;
  check(fn_->dataset_batch(ctx_, indices.data(), (int32_t)indices.size(), &in, &tg));
  return {wrap(in), wrap(tg)};
}

void NativeBackend::dataset_close() {
  if (fn_->dataset_close) check(fn_->dataset_close(ctx_));
}

Tensor NativeBackend::wrap(const pai_tensor& d) {
  auto st = std::make_shared<Storage>();
  st->backend = this;
  live_.insert(st.get());
  st->base = d.base;
  st->count = 1;
  for (int i = 0; i < d.rank; i++) st->count *= d.dims[i];
  if (!scopes_.empty()) {
    st->scope = (int)scopes_.size() - 1;
    scopes_.back().insert(st.get());
  }
  auto t = std::make_shared<TensorImpl>();
  t->shape.assign(d.dims, d.dims + d.rank);
  t->strides.assign(d.strides, d.strides + d.rank);
  t->offset = d.offset;
  t->storage = st;
  return t;
}

void NativeBackend::free_storage(Storage* s) {
  if (s->freed) return;
  s->freed = true;
  if (s->scope >= 0 && s->scope < (int)scopes_.size()) scopes_[(size_t)s->scope].erase(s);
  // Dead views free their block at once; reuse is ordered on the backend's stream, so kernels still reading it
  // finish first.
  if (ctx_) fn_->release(ctx_, s->base);
}

void NativeBackend::invalidate_shadow(const Tensor& t) {
  if (t->storage) t->storage->shadow.reset();
  t->known.reset();
}

Tensor NativeBackend::allocate(const Dims& shape) {
  std::vector<int32_t> d(shape.begin(), shape.end());
  pai_tensor out;
  check(fn_->alloc(ctx_, (int32_t)d.size(), d.data(), PAI_F32, &out));
  Tensor t = wrap(out);
  if (t->numel() == 1) t->known = 0.0f;
  return t;
}

Tensor NativeBackend::from_host(const float* data, int64_t count, const Dims& shape) {
  std::vector<int32_t> d(shape.begin(), shape.end());
  pai_tensor out;
  check(fn_->from_host(ctx_, data, count, (int32_t)d.size(), d.data(), PAI_F32, &out));
  Tensor t = wrap(out);
  int64_t n = t->numel();
  if (n <= (1 << 20)) t->storage->shadow = std::make_shared<std::vector<float>>(data, data + n);
  if (n == 1) t->known = data[0];
  return t;
}

void NativeBackend::to_host(const Tensor& t, float* dst, int64_t count) {
  int64_t n = t->numel();
  if (count < n) throw ArgumentError("ToHost: destination too small");
  if (t->known && n == 1) { dst[0] = *t->known; return; }
  if (t->storage && t->storage->shadow && !t->storage->freed) {
    const auto& sh = *t->storage->shadow;
    // Gather the view's logical elements from the host copy (Tensor.EnumerateOffsets order).
    std::vector<int> ctr((size_t)t->rank(), 0);
    for (int64_t i = 0; i < n; i++) {
      int64_t off = t->offset;
      for (int a = 0; a < t->rank(); a++) off += ctr[(size_t)a] * t->strides[(size_t)a];
      dst[i] = sh[(size_t)off];
      for (int a = t->rank() - 1; a >= 0; a--) {
        if (++ctr[(size_t)a] < t->shape[(size_t)a]) break;
        ctr[(size_t)a] = 0;
      }
    }
    return;
  }
  pai_tensor d = t->desc();
  check(fn_->to_host(ctx_, &d, dst, count));
}

void NativeBackend::copy(const Tensor& src, const Tensor& dst) {
  pai_tensor s = src->desc(), d = dst->desc();
  check(fn_->copy(ctx_, &s, &d));
  invalidate_shadow(dst);
}

enum { kAdd, kSub, kMul, kDiv, kAddS, kMulS, kSqrt, kSigmoid, kSilu, kSum, kMean, kMax };

Tensor NativeBackend::binary(int which, const Tensor& a, const Tensor& b) {
  pai_tensor da = a->desc(), db = b->desc(), out;
  switch (which) {
    case kAdd: check(fn_->add(ctx_, &da, &db, &out)); break;
    case kSub: check(fn_->sub(ctx_, &da, &db, &out)); break;
    case kMul: check(fn_->mul(ctx_, &da, &db, &out)); break;
    default: check(fn_->div(ctx_, &da, &db, &out)); break;
  }
  Tensor r = wrap(out);
  if (r->numel() == 1 && a->known && b->known) {
    float x = *a->known, y = *b->known;
    r->known = which == kAdd ? x + y : which == kSub ? x - y : which == kMul ? x * y : x / y;
  }
  return r;
}

Tensor NativeBackend::unary(int which, const Tensor& x, float s) {
  pai_tensor dx = x->desc(), out;
  switch (which) {
    case kAddS: check(fn_->add_scalar(ctx_, &dx, s, &out)); break;
    case kMulS: check(fn_->mul_scalar(ctx_, &dx, s, &out)); break;
    case kSqrt: check(fn_->sqrt(ctx_, &dx, &out)); break;
    case kSigmoid: check(fn_->sigmoid(ctx_, &dx, &out)); break;
    default: check(fn_->silu(ctx_, &dx, &out)); break;
  }
  Tensor r = wrap(out);
  if (r->numel() == 1 && x->known && (which == kAddS || which == kMulS))
    r->known = which == kAddS ? *x->known + s : *x->known * s;
  return r;
}

Tensor NativeBackend::reduce(int which, const Tensor& x, int axis, bool keep) {
  pai_tensor dx = x->desc(), out;
  switch (which) {
    case kSum: check(fn_->sum(ctx_, &dx, axis, keep, &out)); break;
    case kMean: check(fn_->mean(ctx_, &dx, axis, keep, &out)); break;
    default: check(fn_->max(ctx_, &dx, axis, keep, &out)); break;
  }
  Tensor r = wrap(out);
  if (x->numel() == 1 && x->known) r->known = x->known;  // reducing a single element leaves it unchanged
  return r;
}

Tensor NativeBackend::add(const Tensor& a, const Tensor& b) { return binary(kAdd, a, b); }
Tensor NativeBackend::sub(const Tensor& a, const Tensor& b) { return binary(kSub, a, b); }
Tensor NativeBackend::mul(const Tensor& a, const Tensor& b) { return binary(kMul, a, b); }
Tensor NativeBackend::div(const Tensor& a, const Tensor& b) { return binary(kDiv, a, b); }
Tensor NativeBackend::add_scalar(const Tensor& a, float s) { return unary(kAddS, a, s); }
Tensor NativeBackend::mul_scalar(const Tensor& a, float s) { return unary(kMulS, a, s); }
Tensor NativeBackend::sqrt(const Tensor& x) { return unary(kSqrt, x); }
Tensor NativeBackend::sigmoid(const Tensor& x) { return unary(kSigmoid, x); }
Tensor NativeBackend::silu(const Tensor& x) { return unary(kSilu, x); }
Tensor NativeBackend::sum(const Tensor& x, int axis, bool keep) { return reduce(kSum, x, axis, keep); }
Tensor NativeBackend::mean(const Tensor& x, int axis, bool keep) { return reduce(kMean, x, axis, keep); }
Tensor NativeBackend::max(const Tensor& x, int axis, bool keep) { return reduce(kMax, x, axis, keep); }

Tensor NativeBackend::matmul(const Tensor& a, const Tensor& b, bool tb) {
  pai_tensor da = a->desc(), db = b->desc(), out;
  check(fn_->matmul(ctx_, &da, &db, tb ? 1 : 0, &out));
  return wrap(out);
}

Tensor NativeBackend::softmax(const Tensor& x, int axis) {
  pai_tensor dx = x->desc(), out;
  check(fn_->softmax(ctx_, &dx, axis, &out));
  return wrap(out);
}

Tensor NativeBackend::rms_norm(const Tensor& x, const Tensor& w, float eps) {
  pai_tensor dx = x->desc(), dw = w->desc(), out;
  check(fn_->rmsnorm(ctx_, &dx, &dw, eps, &out));
  return wrap(out);
}

Tensor NativeBackend::rotary(const Tensor& x, const Tensor& c, const Tensor& s) {
  pai_tensor dx = x->desc(), dc = c->desc(), ds = s->desc(), out;
  check(fn_->rotary(ctx_, &dx, &dc, &ds, &out));
  return wrap(out);
}

Tensor NativeBackend::gather(const Tensor& table, const std::vector<int>& ids) {
  pai_tensor dt = table->desc(), out;
  check(fn_->gather(ctx_, &dt, ids.data(), (int64_t)ids.size(), &out));
  return wrap(out);
}

Tensor NativeBackend::scatter_add_rows(const Tensor& rows, const std::vector<int>& ids, int row_count) {
  pai_tensor dr = rows->desc(), out;
  check(fn_->scatter_add_rows(ctx_, &dr, ids.data(), (int64_t)ids.size(), row_count, &out));
  return wrap(out);
}

Tensor NativeBackend::cross_entropy(const Tensor& logits, const std::vector<int>& t, int ignore) {
  pai_tensor dl = logits->desc(), out;
  check(fn_->cross_entropy(ctx_, &dl, t.data(), (int64_t)t.size(), ignore, &out));
  return wrap(out);
}

Tensor NativeBackend::cross_entropy_grad(const Tensor& logits, const std::vector<int>& t, int ignore) {
  pai_tensor dl = logits->desc(), out;
  check(fn_->cross_entropy_grad(ctx_, &dl, t.data(), (int64_t)t.size(), ignore, &out));
  return wrap(out);
}

Tensor NativeBackend::cat(const Tensor& a, const Tensor& b, int axis) {
  pai_tensor da = a->desc(), db = b->desc(), out;
  check(fn_->cat(ctx_, &da, &db, axis, &out));
  return wrap(out);
}

std::pair<Tensor, Tensor> NativeBackend::sdpa_fwd(const Tensor& q, const Tensor& k, const Tensor& v, float scale, bool causal,
                                                  int pos) {
  pai_tensor dq = q->desc(), dk = k->desc(), dv = v->desc(), o, l;
  check(fn_->sdpa_fwd(ctx_, &dq, &dk, &dv, scale, causal ? 1 : 0, pos, &o, &l));
  Tensor to = wrap(o);
  Tensor tl = wrap(l);
  return {to, tl};
}

std::vector<Tensor> NativeBackend::sdpa_bwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o,
                                            const Tensor& lse, const Tensor& dout, float scale, bool causal, int pos) {
  pai_tensor dq = q->desc(), dk = k->desc(), dv = v->desc(), dO = o->desc(), dl = lse->desc(), dd = dout->desc(), r1, r2, r3;
  check(fn_->sdpa_bwd(ctx_, &dq, &dk, &dv, &dO, &dl, &dd, scale, causal ? 1 : 0, pos, &r1, &r2, &r3));
  Tensor a = wrap(r1);
  Tensor b = wrap(r2);
  Tensor c = wrap(r3);
  return {a, b, c};
}

std::pair<Tensor, Tensor> NativeBackend::rms_norm_bwd(const Tensor& x, const Tensor& w, const Tensor& g, float eps) {
  pai_tensor dx = x->desc(), dw = w->desc(), dg = g->desc(), r1, r2;
  check(fn_->rmsnorm_bwd(ctx_, &dx, &dw, &dg, eps, &r1, &r2));
  Tensor a = wrap(r1);
  Tensor b = wrap(r2);
  return {a, b};
}

Tensor NativeBackend::silu_mul(const Tensor& gate, const Tensor& up) {
  pai_tensor dg = gate->desc(), du = up->desc(), out;
  check(fn_->silu_mul_fwd(ctx_, &dg, &du, &out));
  return wrap(out);
}

std::pair<Tensor, Tensor> NativeBackend::silu_mul_bwd(const Tensor& gate, const Tensor& up, const Tensor& g) {
  pai_tensor dg = gate->desc(), du = up->desc(), dd = g->desc(), r1, r2;
  check(fn_->silu_mul_bwd(ctx_, &dg, &du, &dd, &r1, &r2));
  Tensor a = wrap(r1);
  Tensor b = wrap(r2);
  return {a, b};
}

std::pair<Tensor, Tensor> NativeBackend::cross_entropy_fused(const Tensor& logits, const std::vector<int>& t, int ignore,
                                                             float scale) {
  pai_tensor dl = logits->desc(), r1, r2;
  check(fn_->cross_entropy_fused(ctx_, &dl, t.data(), (int64_t)t.size(), ignore, scale, &r1, &r2));
  Tensor a = wrap(r1);
  Tensor b = wrap(r2);
  return {a, b};
}

void NativeBackend::adamw_step(const Tensor& p, const Tensor& g, const Tensor& m, const Tensor& v, float lr, float b1,
                               float b2, float eps, float wd, int t, float grad_scale) {
  pai_tensor dp = p->desc(), dg = g->desc(), dm = m->desc(), dv = v->desc();
  check(fn_->adamw_step(ctx_, &dp, &dg, &dm, &dv, lr, b1, b2, eps, wd, t, grad_scale));
  invalidate_shadow(p);
}

void NativeBackend::begin_scope() {
  check(fn_->scope_begin(ctx_));
  scopes_.emplace_back();
}

void NativeBackend::end_scope() {
  if (scopes_.empty()) throw InvalidOperationError("EndScope without an open scope");
  auto owned = std::move(scopes_.back());
  scopes_.pop_back();
  for (Storage* s : owned) s->freed = true;  // the native scope frees their blocks
  check(fn_->scope_end(ctx_));
}

void NativeBackend::keep_alive(const Tensor& t) {
  Storage* s = t->storage.get();
  if (!s || s->freed) throw InvalidOperationError("KeepAlive of a released tensor");
  check(fn_->keep_alive(ctx_, s->base));
  if (s->scope < 0) return;
  scopes_[(size_t)s->scope].erase(s);
  s->scope -= 1;
  if (s->scope >= 0) scopes_[(size_t)s->scope].insert(s);
}

void NativeBackend::release(const Tensor& t) {
  Storage* s = t->storage.get();
  if (!s || s->freed) return;
  free_storage(s);
}

void NativeBackend::sync() { check(fn_->sync(ctx_)); }

void NativeBackend::memory_stats(int64_t* in_use, int64_t* peak, int64_t* reserved) {
  check(fn_->memory_stats(ctx_, in_use, peak, reserved));
}

void NativeBackend::reset_peak() { check(fn_->reset_peak(ctx_)); }

void NativeBackend::nccl_unique_id(uint8_t out[128]) {
  if (!fn_->nccl_unique_id) throw BackendError("backend has no data-parallel support");
  check(fn_->nccl_unique_id(out));
}

void NativeBackend::nccl_init(const uint8_t id[128], int rank, int world, int timeout_ms) {
  if (!has_dp()) throw BackendError("backend has no data-parallel support");
  check(fn_->nccl_init(ctx_, id, rank, world, timeout_ms));
  dp_rank = rank;
  dp_world = world;
}

void NativeBackend::allreduce(const std::vector<Tensor>& grads) {
  if (dp_world <= 1 || grads.empty()) return;
  std::vector<pai_tensor> d;
  d.reserve(grads.size());
  for (const auto& g : grads) d.push_back(g->desc());
  check(fn_->allreduce_bucket(ctx_, d.data(), (int32_t)d.size()));
}

void NativeBackend::nccl_abort() {
  if (fn_->nccl_abort) check(fn_->nccl_abort(ctx_));
}

void NativeBackend::reduce_scatter(const std::vector<Tensor>& grads) {
  if (dp_world <= 1 || grads.empty()) return;
  if (!fn_->reduce_scatter_bucket) throw BackendError("backend has no reduce-scatter");
  std::vector<pai_tensor> d;
  for (const auto& g : grads) d.push_back(g->desc());
  check(fn_->reduce_scatter_bucket(ctx_, d.data(), (int32_t)d.size()));
}

void NativeBackend::allgather(const std::vector<Tensor>& params) {
  if (dp_world <= 1 || params.empty()) return;
  if (!fn_->allgather_bucket) throw BackendError("backend has no all-gather");
  std::vector<pai_tensor> d;
  for (const auto& p : params) {
    d.push_back(p->desc());
    invalidate_shadow(p);
  }
  check(fn_->allgather_bucket(ctx_, d.data(), (int32_t)d.size()));
}

std::pair<double, int64_t> NativeBackend::dp_stats() {
  double ms = 0.0;
  int64_t n = 0;
  if (fn_->dp_stats) check(fn_->dp_stats(ctx_, &ms, &n));
  return {ms, n};
}

void NativeBackend::allreduce_wait() {
  if (dp_world <= 1) return;
  check(fn_->allreduce_wait(ctx_));
}

}  // namespace paihost

namespace paihost {

static void need(const void* fn, const char* what) {
  if (!fn) throw BackendError(std::string("backend library does not provide ") + what);
}

void NativeBackend::write(const Tensor& dst, const float* data, int64_t count) {
  need((void*)fn_->write, "write");
  pai_tensor d = dst->desc();
  check(fn_->write(ctx_, data, count, &d));
  invalidate_shadow(dst);
  if (count == 1) dst->known = data[0];
}

Tensor NativeBackend::gather_dev(const Tensor& table, const Tensor& ids) {
  need((void*)fn_->gather_dev, "gather_dev");
  pai_tensor dt = table->desc(), di = ids->desc(), o;
  check(fn_->gather_dev(ctx_, &dt, &di, &o));
  return wrap(o);
}

Tensor NativeBackend::rotary_at(const Tensor& x, const Tensor& cos_table, const Tensor& sin_table, const Tensor& pos) {
  need((void*)fn_->rotary_at, "rotary_at");
  pai_tensor dx = x->desc(), dc = cos_table->desc(), ds = sin_table->desc(), dp = pos->desc(), o;
  check(fn_->rotary_at(ctx_, &dx, &dc, &ds, &dp, &o));
  return wrap(o);
}

void NativeBackend::kv_append(const Tensor& k, const Tensor& v, const Tensor& k_cache, const Tensor& v_cache, const Tensor& pos) {
  need((void*)fn_->kv_append, "kv_append");
  pai_tensor dk = k->desc(), dv = v->desc(), dkc = k_cache->desc(), dvc = v_cache->desc(), dp = pos->desc();
  check(fn_->kv_append(ctx_, &dk, &dv, &dkc, &dvc, &dp));
  invalidate_shadow(k_cache);
  invalidate_shadow(v_cache);
}

Tensor NativeBackend::sdpa_decode(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache, const Tensor& pos, float scale) {
  need((void*)fn_->sdpa_decode, "sdpa_decode");
  pai_tensor dq = q->desc(), dk = k_cache->desc(), dv = v_cache->desc(), dp = pos->desc(), o;
  check(fn_->sdpa_decode(ctx_, &dq, &dk, &dv, &dp, scale, &o));
  return wrap(o);
}

Tensor NativeBackend::argmax_rows(const Tensor& x) {
  need((void*)fn_->argmax_rows, "argmax_rows");
  pai_tensor dx = x->desc(), o;
  check(fn_->argmax_rows(ctx_, &dx, &o));
  return wrap(o);
}

Tensor NativeBackend::linear_fused(const Tensor& x, const std::vector<Tensor>& weights, int mode, const Tensor& residual,
                                   const Tensor& norm_weight, float eps) {
  need((void*)fn_->linear_fused, "linear_fused");
  pai_tensor dx = x->desc(), dr{}, dn{};
  std::vector<pai_tensor> dw;
  for (const auto& w : weights) dw.push_back(w->desc());
  if (residual) dr = residual->desc();
  if (norm_weight) dn = norm_weight->desc();
  pai_tensor o;
  check(fn_->linear_fused(ctx_, &dx, norm_weight ? &dn : nullptr, eps, dw.data(), (int32_t)dw.size(), mode,
                          residual ? &dr : nullptr, &o));
  return wrap(o);
}

Tensor NativeBackend::rope_append(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& cos_table,
                                  const Tensor& sin_table, const Tensor& k_cache, const Tensor& v_cache, const Tensor& pos) {
  need((void*)fn_->rope_append, "rope_append");
  pai_tensor dq = q->desc(), dk = k->desc(), dv = v->desc(), dc = cos_table->desc(), ds = sin_table->desc(),
             dkc = k_cache->desc(), dvc = v_cache->desc(), dp = pos->desc(), o;
  check(fn_->rope_append(ctx_, &dq, &dk, &dv, &dc, &ds, &dkc, &dvc, &dp, &o));
  invalidate_shadow(k_cache);
  invalidate_shadow(v_cache);
  return wrap(o);
}

Tensor NativeBackend::attn_decode_step(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& cos_table,
                                       const Tensor& sin_table, const Tensor& k_cache, const Tensor& v_cache, const Tensor& pos,
                                       float scale) {
  need((void*)fn_->attn_decode_step, "attn_decode_step");
  pai_tensor dq = q->desc(), dk = k->desc(), dv = v->desc(), dc = cos_table->desc(), ds = sin_table->desc(),
             dkc = k_cache->desc(), dvc = v_cache->desc(), dp = pos->desc(), o;
  check(fn_->attn_decode_step(ctx_, &dq, &dk, &dv, &dc, &ds, &dkc, &dvc, &dp, scale, &o));
  invalidate_shadow(k_cache);
  invalidate_shadow(v_cache);
  return wrap(o);
}

void NativeBackend::graph_begin() { need((void*)fn_->graph_begin, "graph_begin"); check(fn_->graph_begin(ctx_)); }

pai_graph* NativeBackend::graph_end() {
  need((void*)fn_->graph_end, "graph_end");
  pai_graph* g = nullptr;
  check(fn_->graph_end(ctx_, &g));
  return g;
}

void NativeBackend::graph_launch(pai_graph* g) { need((void*)fn_->graph_launch, "graph_launch"); check(fn_->graph_launch(ctx_, g)); }

void NativeBackend::graph_destroy(pai_graph* g) {
  if (g && fn_->graph_destroy) check(fn_->graph_destroy(ctx_, g));
}

void NativeBackend::timer_start() { need((void*)fn_->timer_start, "timer_start"); check(fn_->timer_start(ctx_)); }

float NativeBackend::timer_stop() {
  need((void*)fn_->timer_stop, "timer_stop");
  float ms = 0;
  check(fn_->timer_stop(ctx_, &ms));
  return ms;
}

int64_t NativeBackend::launch_count() {
  need((void*)fn_->launch_count, "launch_count");
  int64_t n = 0;
  check(fn_->launch_count(ctx_, &n));
  return n;
}

void NativeBackend::kernel_timing(bool on) { need((void*)fn_->kernel_timing, "kernel_timing"); check(fn_->kernel_timing(ctx_, on ? 1 : 0)); }

void NativeBackend::kernel_stats(const std::string& family, int64_t* launches, double* ms, double* work) {
  need((void*)fn_->kernel_stats, "kernel_stats");
  check(fn_->kernel_stats(ctx_, family.c_str(), launches, ms, work));
}

void NativeBackend::check_device_error() {
  if (!fn_->check_device_error) return;
  int32_t code = 0;
  check(fn_->check_device_error(ctx_, &code));
}

}  // namespace paihost
