// ORACLE — test infrastructure only. A CPU restatement of project-ai's CpuComputeBackend
// (ProjectAI.Backends.Cpu/CpuComputeBackend.cs), exported through the same C ABI as libprojectai_cuda.so
// (include/projectai_cuda.h) with the prefix `oracle_` instead of `pai_`. Only the tests, the smoke check
// and the bench's CPU-baseline leg load it; the product never does.
//
// Parity pin: the reference is C#/.NET and cannot be built or run here (no dotnet). This restatement keeps the
// reference's loop and accumulation orders op by op (each function cites the lines it follows) and is built
// with -O2 -fno-fast-math -ffp-contract=off so every float operation rounds exactly as the IEEE single
// operations of the C# code do (CoreCLR does not contract a*b+c). MathF.Exp/Sqrt/Log/Pow/Sin/Cos map to glibc
// expf/sqrtf/logf/powf/sinf/cosf; Math.Exp/Log to exp/log. It is pinned against the reference's own
// known-answer tests (tests/test_oracle_golden.py).
//
// Threads: oracle_set_threads(n) lets loops over independent output elements run in parallel (OpenMP). Each
// output element keeps its sequential accumulation order, and cross-row sums (the cross-entropy total) are
// reduced in row order afterwards, so results are bit-identical for every thread count.
#include "projectai_cuda.h"

#include <cerrno>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_err = "";

pai_status fail(pai_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return st;
}

int g_threads = 1;

struct Block { int64_t count; int scope; };  // scope = -1: owned by no scope

}  // namespace

struct pai_ctx {
  std::unordered_map<void*, Block> blocks;
  std::vector<std::unordered_set<void*>> scopes;
  int64_t in_use = 0, peak = 0;
  // the open packed dataset (oracle_dataset_open): its blocks' bytes, id width, sequence length, block count
  std::vector<uint8_t> ds_bytes;
  int ds_elem = 0, ds_seq = 0;
  int64_t ds_blocks = 0;
  // the last checkpoint read by oracle_ckpt_load
  std::string ck_meta;
  std::vector<std::string> ck_names;
  std::vector<pai_tensor> ck_tensors;
};

namespace {

#define CHECK_CTX(c) do { if (!(c)) return fail(PAI_ERR_ARGUMENT, "null context"); } while (0)
#define TRY(x) do { pai_status _s = (x); if (_s != PAI_OK) return _s; } while (0)

int64_t numel(const pai_tensor& t) {
  int64_t n = 1;
  for (int i = 0; i < t.rank; i++) n *= t.dims[i];
  return n;
}

std::string shape_str(const pai_tensor& t) {
  std::string s = "[";
  for (int i = 0; i < t.rank; i++) { if (i) s += ", "; s += std::to_string(t.dims[i]); }
  return s + "]";
}

void set_contig(pai_tensor* t, void* base, int rank, const int32_t* dims, int dtype) {
  memset(t, 0, sizeof *t);
  t->base = base; t->offset = 0; t->rank = rank; t->dtype = dtype;
  int64_t acc = 1;
  for (int i = rank - 1; i >= 0; i--) { t->dims[i] = dims[i]; t->strides[i] = acc; acc *= dims[i]; }
}

pai_status check_desc(pai_ctx* c, const pai_tensor* t, const char* what) {
  if (!t) return fail(PAI_ERR_ARGUMENT, "%s: null tensor", what);
  if (t->rank < 0 || t->rank > PAI_MAX_RANK) return fail(PAI_ERR_ARGUMENT, "%s: rank %d unsupported", what, t->rank);
  auto it = c->blocks.find(t->base);
  if (it == c->blocks.end()) return fail(PAI_ERR_INVALID_OP, "%s: tensor storage is not owned by this backend (freed?)", what);
  // The view must stay inside its storage.
  int64_t lo = t->offset, hi = t->offset;
  for (int i = 0; i < t->rank; i++) {
    if (t->dims[i] < 0) return fail(PAI_ERR_ARGUMENT, "%s: negative dimension", what);
    if (t->dims[i] == 0) return PAI_OK;
    int64_t span = (int64_t)(t->dims[i] - 1) * t->strides[i];
    if (span < 0) lo += span; else hi += span;
  }
  if (lo < 0 || hi >= it->second.count)
    return fail(PAI_ERR_ARGUMENT, "%s: view %s exceeds its storage", what, shape_str(*t).c_str());
  return PAI_OK;
}

pai_status alloc(pai_ctx* c, int rank, const int32_t* dims, int dtype, pai_tensor* out) {
  int64_t n = 1;
  for (int i = 0; i < rank; i++) {
    if (dims[i] < 0) return fail(PAI_ERR_OUT_OF_RANGE, "Dimensions must be non-negative.");
    n *= dims[i];
  }
  // One extra element keeps zero-element tensors distinct and addressable.
  float* p = static_cast<float*>(calloc((size_t)n + 1, sizeof(float)));
  if (!p) return fail(PAI_ERR_OUT_OF_MEMORY, "out of memory allocating %lld floats on the host", (long long)n);
  int scope = c->scopes.empty() ? -1 : (int)c->scopes.size() - 1;
  c->blocks[p] = Block{n, scope};
  if (scope >= 0) c->scopes.back().insert(p);
  c->in_use += n * 4;
  if (c->in_use > c->peak) c->peak = c->in_use;
  set_contig(out, p, rank, dims, dtype);
  return PAI_OK;
}

void free_block(pai_ctx* c, void* p) {
  auto it = c->blocks.find(p);
  if (it == c->blocks.end()) return;
  c->in_use -= it->second.count * 4;
  c->blocks.erase(it);
  free(p);
}

float* buf(const pai_tensor& t) { return static_cast<float*>(t.base); }

// Tensor.EnumerateOffsets (Tensor.cs:173-197): physical offsets in logical row-major order.
template <class F>
void for_each_offset(const pai_tensor& t, F&& f) {
  int64_t total = numel(t);
  if (t.rank == 0) { f((int64_t)0, t.offset); return; }
  int32_t counter[PAI_MAX_RANK] = {0};
  for (int64_t n = 0; n < total; n++) {
    int64_t off = t.offset;
    for (int i = 0; i < t.rank; i++) off += counter[i] * t.strides[i];
    f(n, off);
    for (int ax = t.rank - 1; ax >= 0; ax--) {
      if (++counter[ax] < t.dims[ax]) break;
      counter[ax] = 0;
    }
  }
}

bool is_dense(const pai_tensor& t) {
  int64_t acc = 1;
  for (int i = t.rank - 1; i >= 0; i--) {
    if (t.dims[i] == 1) continue;
    if (t.strides[i] != acc) return false;
    acc *= t.dims[i];
  }
  return true;
}

// A view's logical elements as a dense row-major array: the storage itself when the view is already dense, else a
// gathered copy.
struct Dense {
  std::vector<float> own;
  const float* p = nullptr;
  size_t n = 0;
  float operator[](size_t i) const { return p[i]; }
  size_t size() const { return n; }
  const float* data() const { return p; }
};

// CpuComputeBackend.Materialize (CpuComputeBackend.cs:27-39): the view's logical elements, dense row-major.
Dense materialize(const pai_tensor& t, bool force_copy = false) {
  Dense d;
  d.n = (size_t)numel(t);
  const float* b = buf(t);
  if (is_dense(t) && !force_copy) {
    d.p = b + t.offset;
    return d;
  }
  d.own.resize(d.n);
  for_each_offset(t, [&](int64_t i, int64_t off) { d.own[(size_t)i] = b[off]; });
  d.p = d.own.data();
  return d;
}

// Shape.TryBroadcastWith (Shape.cs:94-113).
bool broadcast_shape(const pai_tensor& a, const pai_tensor& b, int* rank, int32_t* dims) {
  int n = a.rank > b.rank ? a.rank : b.rank;
  for (int i = 0; i < n; i++) {
    int da = i < a.rank ? a.dims[a.rank - 1 - i] : 1;
    int db = i < b.rank ? b.dims[b.rank - 1 - i] : 1;
    int d;
    if (da == db) d = da; else if (da == 1) d = db; else if (db == 1) d = da; else return false;
    dims[n - 1 - i] = d;
  }
  *rank = n;
  return true;
}

// Tensor.BroadcastTo (Tensor.cs:147-168).
pai_tensor broadcast_to(const pai_tensor& t, int rank, const int32_t* dims) {
  pai_tensor r = t;
  int lead = rank - t.rank;
  for (int i = 0; i < rank; i++) {
    r.dims[i] = dims[i];
    if (i < lead) { r.strides[i] = 0; continue; }
    int s = t.dims[i - lead];
    r.strides[i] = (s == dims[i]) ? t.strides[i - lead] : 0;
  }
  r.rank = rank;
  return r;
}

int norm_axis(int axis, int rank) { return axis < 0 ? axis + rank : axis; }

enum BinOp { kAdd, kMul, kSub, kDiv };

// CpuComputeBackend.Elementwise (CpuComputeBackend.cs:93-135). The SIMD fast path and the gather path compute
// the same IEEE single operation per element, so one loop covers both.
pai_status elementwise(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, pai_tensor* out, BinOp op) {
  CHECK_CTX(c);
  TRY(check_desc(c, a, "a"));
  TRY(check_desc(c, b, "b"));
  int rank; int32_t dims[PAI_MAX_RANK];
  if (!broadcast_shape(*a, *b, &rank, dims) || rank > PAI_MAX_RANK)
    return fail(PAI_ERR_ARGUMENT, "Shapes %s and %s are not broadcast-compatible.", shape_str(*a).c_str(), shape_str(*b).c_str());
  pai_tensor av = broadcast_to(*a, rank, dims), bv = broadcast_to(*b, rank, dims);
  pai_tensor r;
  TRY(alloc(c, rank, dims, a->dtype, &r));
  int64_t n = numel(r);
  // Both operands as dense arrays of the result's shape (a broadcast operand is gathered through its stride-0 view).
  Dense da = materialize(av), db = materialize(bv);
  const float* pa = da.data(); const float* pb = db.data(); float* po = buf(r);
#pragma omp parallel for num_threads(g_threads) schedule(static) if (n > 65536)
  for (int64_t i = 0; i < n; i++) {
    float x = pa[i], y = pb[i];
    float z;
    switch (op) {
      case kAdd: z = x + y; break;
      case kMul: z = x * y; break;
      case kSub: z = x - y; break;
      default: z = x / y; break;
    }
    po[i] = z;
  }
  *out = r;
  return PAI_OK;
}

template <class F>
pai_status unary(pai_ctx* c, const pai_tensor* x, pai_tensor* out, F&& f) {
  CHECK_CTX(c);
  TRY(check_desc(c, x, "x"));
  auto src = materialize(*x);
  pai_tensor r;
  TRY(alloc(c, x->rank, x->dims, x->dtype, &r));
  float* po = buf(r);
  int64_t n = (int64_t)src.size();
#pragma omp parallel for num_threads(g_threads) schedule(static) if (n > 65536)
  for (int64_t i = 0; i < n; i++) po[i] = f(src[(size_t)i]);
  *out = r;
  return PAI_OK;
}

// CpuComputeBackend.SigmoidScalar (CpuComputeBackend.cs:312-317): sign-split keeps exp's argument <= 0.
float sigmoid_scalar(float v) {
  if (v >= 0.0f) return 1.0f / (1.0f + expf(-v));
  float t = expf(v);
  return t / (1.0f + t);
}

enum ReduceKind { kSum, kMean, kMax };

// CpuComputeBackend.Reduce (CpuComputeBackend.cs:254-301): layout [outer, axisLen, inner], sequential fp32.
pai_status reduce(pai_ctx* c, const pai_tensor* x, int axis, int keep, pai_tensor* out, ReduceKind kind) {
  CHECK_CTX(c);
  TRY(check_desc(c, x, "x"));
  int rank = x->rank;
  if (rank == 0) return fail(PAI_ERR_ARGUMENT, "Cannot reduce a scalar tensor.");
  int ax = norm_axis(axis, rank);
  if (ax < 0 || ax >= rank) return fail(PAI_ERR_OUT_OF_RANGE, "Axis out of range for shape %s.", shape_str(*x).c_str());
  int64_t outer = 1, inner = 1;
  for (int i = 0; i < ax; i++) outer *= x->dims[i];
  int axis_len = x->dims[ax];
  for (int i = ax + 1; i < rank; i++) inner *= x->dims[i];
  auto src = materialize(*x);
  int32_t odims[PAI_MAX_RANK]; int orank = 0;
  for (int i = 0; i < rank; i++) {
    if (i == ax) { if (keep) odims[orank++] = 1; }
    else odims[orank++] = x->dims[i];
  }
  pai_tensor r;
  TRY(alloc(c, orank, odims, x->dtype, &r));
  float* po = buf(r);
  int64_t total = outer * inner;
#pragma omp parallel for num_threads(g_threads) schedule(static) if (total * axis_len > 65536)
  for (int64_t oc = 0; oc < total; oc++) {
    int64_t o = oc / inner, cc = oc % inner;
    int64_t base = o * axis_len * inner;
    float acc = kind == kMax ? -INFINITY : 0.0f;
    for (int t = 0; t < axis_len; t++) {
      float v = src[(size_t)(base + (int64_t)t * inner + cc)];
      // MathF.Max: NaN if either operand is NaN.
      if (kind == kMax) acc = (std::isnan(acc) || std::isnan(v)) ? NAN : (v > acc ? v : acc);
      else acc = acc + v;
    }
    if (kind == kMean) acc /= (float)axis_len;
    po[o * inner + cc] = acc;
  }
  *out = r;
  return PAI_OK;
}

}  // namespace

ORC_API const char* oracle_last_error(void) { return g_err.c_str(); }

ORC_API void oracle_set_threads(int n) { g_threads = n < 1 ? 1 : n; }

ORC_API pai_status oracle_ctx_create(int device, pai_ctx** out) {
  (void)device;
  if (!out) return fail(PAI_ERR_ARGUMENT, "null out");
  *out = new pai_ctx();
  return PAI_OK;
}

ORC_API pai_status oracle_ctx_destroy(pai_ctx* c) {
  if (!c) return PAI_OK;
  for (auto& kv : c->blocks) free(kv.first);
  delete c;
  return PAI_OK;
}

ORC_API pai_status oracle_sync(pai_ctx* c) { CHECK_CTX(c); return PAI_OK; }

ORC_API pai_status oracle_device_name(pai_ctx* c, char* b, int32_t n) {
  CHECK_CTX(c);
  snprintf(b, (size_t)n, "cpu-reference");
  return PAI_OK;
}

// CpuComputeBackend.Allocate (CpuComputeBackend.cs:41-42): zeroed.
ORC_API pai_status oracle_alloc(pai_ctx* c, int32_t rank, const int32_t* dims, int32_t dtype, pai_tensor* out) {
  CHECK_CTX(c);
  if (rank < 0 || rank > PAI_MAX_RANK) return fail(PAI_ERR_ARGUMENT, "rank %d unsupported", rank);
  return alloc(c, rank, dims, dtype, out);
}

// CpuComputeBackend.FromHost (CpuComputeBackend.cs:44-49).
ORC_API pai_status oracle_from_host(pai_ctx* c, const float* host, int64_t count, int32_t rank, const int32_t* dims,
                                    int32_t dtype, pai_tensor* out) {
  CHECK_CTX(c);
  if (rank < 0 || rank > PAI_MAX_RANK) return fail(PAI_ERR_ARGUMENT, "rank %d unsupported", rank);
  pai_tensor r;
  TRY(alloc(c, rank, dims, dtype, &r));
  if (count < numel(r)) return fail(PAI_ERR_ARGUMENT, "FromHost: %lld values for %lld elements", (long long)count, (long long)numel(r));
  if (numel(r)) memcpy(r.base, host, (size_t)numel(r) * 4);
  *out = r;
  return PAI_OK;
}

// CpuComputeBackend.ToHost (CpuComputeBackend.cs:55-67).
ORC_API pai_status oracle_to_host(pai_ctx* c, const pai_tensor* src, float* host, int64_t count) {
  CHECK_CTX(c);
  TRY(check_desc(c, src, "source"));
  if (count < numel(*src)) return fail(PAI_ERR_ARGUMENT, "ToHost: destination too small");
  const float* b = buf(*src);
  for_each_offset(*src, [&](int64_t i, int64_t off) { host[i] = b[off]; });
  return PAI_OK;
}

// CpuComputeBackend.Copy (CpuComputeBackend.cs:69-81).
ORC_API pai_status oracle_copy(pai_ctx* c, const pai_tensor* src, const pai_tensor* dst) {
  CHECK_CTX(c);
  TRY(check_desc(c, src, "source"));
  TRY(check_desc(c, dst, "destination"));
  if (numel(*src) != numel(*dst)) return fail(PAI_ERR_ARGUMENT, "Copy: element counts differ (%s vs %s)", shape_str(*src).c_str(), shape_str(*dst).c_str());
  auto s = materialize(*src, src->base == dst->base);  // a copy within one storage reads a snapshot
  float* d = buf(*dst);
  for_each_offset(*dst, [&](int64_t i, int64_t off) { d[off] = s[(size_t)i]; });
  return PAI_OK;
}

ORC_API pai_status oracle_scope_begin(pai_ctx* c) {
  CHECK_CTX(c);
  c->scopes.emplace_back();
  return PAI_OK;
}

ORC_API pai_status oracle_scope_end(pai_ctx* c) {
  CHECK_CTX(c);
  if (c->scopes.empty()) return fail(PAI_ERR_INVALID_OP, "scope_end without an open scope");
  auto owned = std::move(c->scopes.back());
  c->scopes.pop_back();
  for (void* p : owned) free_block(c, p);
  return PAI_OK;
}

// KeepAlive promotes out of exactly one scope (IComputeBackend.cs:80-87).
ORC_API pai_status oracle_keep_alive(pai_ctx* c, const void* base) {
  CHECK_CTX(c);
  void* p = const_cast<void*>(base);
  auto it = c->blocks.find(p);
  if (it == c->blocks.end()) return fail(PAI_ERR_INVALID_OP, "KeepAlive of a tensor this backend does not own");
  int s = it->second.scope;
  if (s < 0) return PAI_OK;
  c->scopes[(size_t)s].erase(p);
  int parent = s - 1;
  it->second.scope = parent;
  if (parent >= 0) c->scopes[(size_t)parent].insert(p);
  return PAI_OK;
}

ORC_API pai_status oracle_release(pai_ctx* c, const void* base) {
  CHECK_CTX(c);
  void* p = const_cast<void*>(base);
  auto it = c->blocks.find(p);
  if (it == c->blocks.end()) return PAI_OK;
  if (it->second.scope >= 0) c->scopes[(size_t)it->second.scope].erase(p);
  free_block(c, p);
  return PAI_OK;
}

ORC_API pai_status oracle_finalize(pai_ctx* c, const void* base) {
  CHECK_CTX(c);
  void* p = const_cast<void*>(base);
  auto it = c->blocks.find(p);
  if (it == c->blocks.end() || it->second.scope >= 0) return PAI_OK;
  free_block(c, p);
  return PAI_OK;
}

ORC_API pai_status oracle_memory_stats(pai_ctx* c, int64_t* in_use, int64_t* peak, int64_t* reserved) {
  CHECK_CTX(c);
  if (in_use) *in_use = c->in_use;
  if (peak) *peak = c->peak;
  if (reserved) *reserved = c->in_use;
  return PAI_OK;
}

ORC_API pai_status oracle_reset_peak(pai_ctx* c) { CHECK_CTX(c); c->peak = c->in_use; return PAI_OK; }

ORC_API pai_status oracle_add(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, pai_tensor* o) { return elementwise(c, a, b, o, kAdd); }
ORC_API pai_status oracle_sub(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, pai_tensor* o) { return elementwise(c, a, b, o, kSub); }
ORC_API pai_status oracle_mul(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, pai_tensor* o) { return elementwise(c, a, b, o, kMul); }
ORC_API pai_status oracle_div(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, pai_tensor* o) { return elementwise(c, a, b, o, kDiv); }

// CpuComputeBackend.AddScalar/MulScalar/Sqrt (CpuComputeBackend.cs:137-156).
ORC_API pai_status oracle_add_scalar(pai_ctx* c, const pai_tensor* a, float s, pai_tensor* o) {
  return unary(c, a, o, [s](float v) { return v + s; });
}
ORC_API pai_status oracle_mul_scalar(pai_ctx* c, const pai_tensor* a, float s, pai_tensor* o) {
  return unary(c, a, o, [s](float v) { return v * s; });
}
ORC_API pai_status oracle_sqrt(pai_ctx* c, const pai_tensor* x, pai_tensor* o) {
  return unary(c, x, o, [](float v) { return sqrtf(v); });
}
// CpuComputeBackend.Sigmoid (CpuComputeBackend.cs:304-310).
ORC_API pai_status oracle_sigmoid(pai_ctx* c, const pai_tensor* x, pai_tensor* o) {
  return unary(c, x, o, [](float v) { return sigmoid_scalar(v); });
}
// CpuComputeBackend.Silu (CpuComputeBackend.cs:385-391).
ORC_API pai_status oracle_silu(pai_ctx* c, const pai_tensor* x, pai_tensor* o) {
  return unary(c, x, o, [](float v) { return v * sigmoid_scalar(v); });
}

// CpuComputeBackend.MatMul (CpuComputeBackend.cs:159-219): batch broadcast, sequential fp32 dot products.
ORC_API pai_status oracle_matmul(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, int32_t tb, pai_tensor* out) {
  CHECK_CTX(c);
  TRY(check_desc(c, a, "a"));
  TRY(check_desc(c, b, "b"));
  int ra = a->rank, rb = b->rank;
  if (ra < 2 || rb < 2)
    return fail(PAI_ERR_ARGUMENT, "MatMul requires rank >= 2 operands; got %s and %s.", shape_str(*a).c_str(), shape_str(*b).c_str());
  int m = a->dims[ra - 2], k = a->dims[ra - 1];
  int kb = tb ? b->dims[rb - 1] : b->dims[rb - 2];
  int n = tb ? b->dims[rb - 2] : b->dims[rb - 1];
  if (k != kb) return fail(PAI_ERR_ARGUMENT, "MatMul inner dimensions disagree: %s x %s (transposeB=%d).", shape_str(*a).c_str(), shape_str(*b).c_str(), tb);
  pai_tensor ab{}, bb{};
  ab.rank = ra - 2; bb.rank = rb - 2;
  for (int i = 0; i < ra - 2; i++) ab.dims[i] = a->dims[i];
  for (int i = 0; i < rb - 2; i++) bb.dims[i] = b->dims[i];
  int brank; int32_t bdims[PAI_MAX_RANK];
  if (!broadcast_shape(ab, bb, &brank, bdims))
    return fail(PAI_ERR_ARGUMENT, "Shapes %s and %s are not broadcast-compatible.", shape_str(ab).c_str(), shape_str(bb).c_str());
  int64_t batch = 1;
  for (int i = 0; i < brank; i++) batch *= bdims[i];
  auto A = materialize(*a);
  auto B = materialize(*b);
  int64_t ablock = (int64_t)m * k, bblock = (int64_t)kb * n;
  int32_t odims[PAI_MAX_RANK];
  for (int i = 0; i < brank; i++) odims[i] = bdims[i];
  odims[brank] = m; odims[brank + 1] = n;
  if (brank + 2 > PAI_MAX_RANK) return fail(PAI_ERR_ARGUMENT, "MatMul result rank too large");
  pai_tensor r;
  TRY(alloc(c, brank + 2, odims, a->dtype, &r));
  float* po = buf(r);
  // BatchIndex (CpuComputeBackend.cs:222-233): size-1 input batch dims repeat.
  std::vector<int64_t> aoff((size_t)batch), boff((size_t)batch);
  {
    std::vector<int> counter((size_t)brank, 0);
    for (int64_t bi = 0; bi < batch; bi++) {
      int64_t ia = 0, ib = 0;
      int la = brank - ab.rank, lb = brank - bb.rank;
      for (int i = 0; i < ab.rank; i++) ia = ia * ab.dims[i] + (ab.dims[i] == 1 ? 0 : counter[(size_t)(la + i)]);
      for (int i = 0; i < bb.rank; i++) ib = ib * bb.dims[i] + (bb.dims[i] == 1 ? 0 : counter[(size_t)(lb + i)]);
      aoff[(size_t)bi] = ia * ablock; boff[(size_t)bi] = ib * bblock;
      for (int ax = brank - 1; ax >= 0; ax--) { if (++counter[(size_t)ax] < bdims[ax]) break; counter[(size_t)ax] = 0; }
    }
  }
  int64_t rows = batch * m;
#pragma omp parallel for num_threads(g_threads) schedule(static) if (rows * (int64_t)n * k > 65536)
  for (int64_t row = 0; row < rows; row++) {
    int64_t bi = row / m; int i = (int)(row % m);
    int64_t arow = aoff[(size_t)bi] + (int64_t)i * k, bo = boff[(size_t)bi], oo = bi * m * n;
    float* orow = po + oo + (int64_t)i * n;
    if (tb) {
      for (int j = 0; j < n; j++) {
        float acc = 0.0f;
        int64_t brow = bo + (int64_t)j * k;
        for (int p = 0; p < k; p++) acc += A[(size_t)(arow + p)] * B[(size_t)(brow + p)];
        orow[j] = acc;
      }
    } else {
      // Loop order i, p, j: every output element still accumulates its products in p order starting from 0 (the
      // reference's order, CpuComputeBackend.cs:205-208), while B is read along its contiguous rows.
      for (int j = 0; j < n; j++) orow[j] = 0.0f;
      for (int p = 0; p < k; p++) {
        float av = A[(size_t)(arow + p)];
        const float* brow = B.data() + bo + (int64_t)p * n;
        for (int j = 0; j < n; j++) orow[j] += av * brow[j];
      }
    }
  }
  *out = r;
  return PAI_OK;
}

ORC_API pai_status oracle_sum(pai_ctx* c, const pai_tensor* x, int32_t axis, int32_t keep, pai_tensor* o) { return reduce(c, x, axis, keep, o, kSum); }
ORC_API pai_status oracle_mean(pai_ctx* c, const pai_tensor* x, int32_t axis, int32_t keep, pai_tensor* o) { return reduce(c, x, axis, keep, o, kMean); }
ORC_API pai_status oracle_max(pai_ctx* c, const pai_tensor* x, int32_t axis, int32_t keep, pai_tensor* o) { return reduce(c, x, axis, keep, o, kMax); }

// CpuComputeBackend.Softmax (CpuComputeBackend.cs:322-358).
ORC_API pai_status oracle_softmax(pai_ctx* c, const pai_tensor* x, int32_t axis, pai_tensor* out) {
  CHECK_CTX(c);
  TRY(check_desc(c, x, "x"));
  int rank = x->rank;
  if (rank == 0) return fail(PAI_ERR_ARGUMENT, "Softmax requires rank >= 1.");
  int ax = norm_axis(axis, rank);
  if (ax < 0 || ax >= rank) return fail(PAI_ERR_OUT_OF_RANGE, "Specified argument was out of the range of valid values. (Parameter 'axis')");
  int64_t outer = 1, inner = 1;
  for (int i = 0; i < ax; i++) outer *= x->dims[i];
  int len = x->dims[ax];
  for (int i = ax + 1; i < rank; i++) inner *= x->dims[i];
  auto src = materialize(*x);
  pai_tensor r;
  TRY(alloc(c, rank, x->dims, x->dtype, &r));
  float* dst = buf(r);
  int64_t total = outer * inner;
#pragma omp parallel for num_threads(g_threads) schedule(static) if (total * len > 65536)
  for (int64_t oc = 0; oc < total; oc++) {
    int64_t o = oc / inner, cc = oc % inner;
    int64_t b = o * len * inner + cc;
    float mx = -INFINITY;
    for (int k = 0; k < len; k++) { float v = src[(size_t)(b + (int64_t)k * inner)]; if (v > mx) mx = v; }
    float sum = 0.0f;
    for (int k = 0; k < len; k++) {
      float e = expf(src[(size_t)(b + (int64_t)k * inner)] - mx);
      dst[b + (int64_t)k * inner] = e;
      sum += e;
    }
    float inv = 1.0f / sum;
    for (int k = 0; k < len; k++) dst[b + (int64_t)k * inner] *= inv;
  }
  *out = r;
  return PAI_OK;
}

// CpuComputeBackend.RmsNorm (CpuComputeBackend.cs:361-382).
ORC_API pai_status oracle_rmsnorm(pai_ctx* c, const pai_tensor* x, const pai_tensor* w, float eps, pai_tensor* out) {
  CHECK_CTX(c);
  TRY(check_desc(c, x, "x"));
  TRY(check_desc(c, w, "weight"));
  int rank = x->rank;
  if (rank == 0) return fail(PAI_ERR_ARGUMENT, "RmsNorm requires rank >= 1.");
  int d = x->dims[rank - 1];
  if (w->rank != 1 || w->dims[0] != d)
    return fail(PAI_ERR_ARGUMENT, "RmsNorm weight must be [%d] to match the last axis of %s.", d, shape_str(*x).c_str());
  auto src = materialize(*x);
  auto wv = materialize(*w);
  pai_tensor r;
  TRY(alloc(c, rank, x->dims, x->dtype, &r));
  float* dst = buf(r);
  int64_t rows = d ? numel(*x) / d : 0;
#pragma omp parallel for num_threads(g_threads) schedule(static) if (rows * d > 65536)
  for (int64_t row = 0; row < rows; row++) {
    int64_t b = row * d;
    float ss = 0.0f;
    for (int j = 0; j < d; j++) { float v = src[(size_t)(b + j)]; ss += v * v; }
    float inv = 1.0f / sqrtf(ss / (float)d + eps);
    for (int j = 0; j < d; j++) dst[b + j] = src[(size_t)(b + j)] * inv * wv[(size_t)j];
  }
  *out = r;
  return PAI_OK;
}

// CpuComputeBackend.RotaryEmbedding (CpuComputeBackend.cs:397-420).
ORC_API pai_status oracle_rotary(pai_ctx* c, const pai_tensor* x, const pai_tensor* cs, const pai_tensor* sn, pai_tensor* out) {
  CHECK_CTX(c);
  TRY(check_desc(c, x, "x"));
  TRY(check_desc(c, cs, "cos"));
  TRY(check_desc(c, sn, "sin"));
  int rank = x->rank;
  if (rank == 0) return fail(PAI_ERR_ARGUMENT, "RotaryEmbedding requires rank >= 1.");
  int d = x->dims[rank - 1];
  if (d % 2) return fail(PAI_ERR_ARGUMENT, "RoPE head dim must be even; got %d.", d);
  int half = d / 2;
  auto check_bcast = [&](const pai_tensor* t) -> bool {
    if (t->rank > rank) return false;
    int lead = rank - t->rank;
    for (int i = 0; i < t->rank; i++) if (t->dims[i] != x->dims[lead + i] && t->dims[i] != 1) return false;
    return true;
  };
  if (!check_bcast(cs) || !check_bcast(sn))
    return fail(PAI_ERR_ARGUMENT, "Cannot broadcast cos/sin to %s.", shape_str(*x).c_str());
  auto src = materialize(*x);
  auto cm = materialize(broadcast_to(*cs, rank, x->dims));
  auto sm = materialize(broadcast_to(*sn, rank, x->dims));
  pai_tensor r;
  TRY(alloc(c, rank, x->dims, x->dtype, &r));
  float* dst = buf(r);
  int64_t rows = d ? numel(*x) / d : 0;
#pragma omp parallel for num_threads(g_threads) schedule(static) if (rows * d > 65536)
  for (int64_t row = 0; row < rows; row++) {
    int64_t b = row * d;
    for (int i = 0; i < d; i++) {
      float rot = i < half ? -src[(size_t)(b + i + half)] : src[(size_t)(b + i - half)];
      dst[b + i] = src[(size_t)(b + i)] * cm[(size_t)(b + i)] + rot * sm[(size_t)(b + i)];
    }
  }
  *out = r;
  return PAI_OK;
}

// CpuComputeBackend.Gather (CpuComputeBackend.cs:424-436).
ORC_API pai_status oracle_gather(pai_ctx* c, const pai_tensor* table, const int32_t* ids, int64_t n, pai_tensor* out) {
  CHECK_CTX(c);
  TRY(check_desc(c, table, "table"));
  if (table->rank != 2) return fail(PAI_ERR_ARGUMENT, "Gather: table must be [vocab, dim]");
  int vocab = table->dims[0], dim = table->dims[1];
  auto src = materialize(*table);
  for (int64_t i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= vocab)
      return fail(PAI_ERR_OUT_OF_RANGE, "id out of range [0,%d). (Parameter 'ids') Actual value was %d.", vocab, ids[i]);
  int32_t od[2] = {(int32_t)n, dim};
  pai_tensor r;
  TRY(alloc(c, 2, od, table->dtype, &r));
  float* dst = buf(r);
  for (int64_t i = 0; i < n; i++) memcpy(dst + i * dim, src.data() + (int64_t)ids[i] * dim, (size_t)dim * 4);
  *out = r;
  return PAI_OK;
}

// CpuComputeBackend.ScatterAddRows (CpuComputeBackend.cs:438-451): sequential per-id row adds.
ORC_API pai_status oracle_scatter_add_rows(pai_ctx* c, const pai_tensor* rows, const int32_t* ids, int64_t n,
                                          int32_t row_count, pai_tensor* out) {
  CHECK_CTX(c);
  TRY(check_desc(c, rows, "rows"));
  if (rows->rank < 1) return fail(PAI_ERR_ARGUMENT, "ScatterAddRows: rows must have rank >= 1");
  int dim = rows->dims[rows->rank - 1];
  auto src = materialize(*rows);
  if ((int64_t)src.size() < n * dim) return fail(PAI_ERR_ARGUMENT, "ScatterAddRows: fewer rows than ids");
  for (int64_t i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= row_count)
      return fail(PAI_ERR_OUT_OF_RANGE, "id out of range [0,%d). (Parameter 'ids') Actual value was %d.", row_count, ids[i]);
  int32_t od[2] = {row_count, dim};
  pai_tensor r;
  TRY(alloc(c, 2, od, rows->dtype, &r));
  float* dst = buf(r);
  for (int64_t i = 0; i < n; i++) {
    int64_t rb = (int64_t)ids[i] * dim, sb = i * dim;
    for (int j = 0; j < dim; j++) dst[rb + j] += src[(size_t)(sb + j)];
  }
  *out = r;
  return PAI_OK;
}

// CpuComputeBackend.CrossEntropy (CpuComputeBackend.cs:453-475): per-row log-sum-exp and the total in double.
ORC_API pai_status oracle_cross_entropy(pai_ctx* c, const pai_tensor* logits, const int32_t* targets, int64_t nt,
                                       int32_t ignore, pai_tensor* out) {
  CHECK_CTX(c);
  TRY(check_desc(c, logits, "logits"));
  if (logits->rank != 2) return fail(PAI_ERR_ARGUMENT, "CrossEntropy: logits must be [N, vocab]");
  int n = logits->dims[0], vocab = logits->dims[1];
  if (nt < n) return fail(PAI_ERR_ARGUMENT, "targets (%lld) must have one entry per logits row (%d).", (long long)nt, n);
  for (int i = 0; i < n; i++) {
    int t = targets[i];
    if (t != ignore && (t < 0 || t >= vocab))
      return fail(PAI_ERR_OUT_OF_RANGE, "target out of range [0,%d). (Parameter 'targets') Actual value was %d.", vocab, t);
  }
  auto src = materialize(*logits);
  std::vector<double> row_loss((size_t)n, 0.0);
#pragma omp parallel for num_threads(g_threads) schedule(static) if ((int64_t)n * vocab > 65536)
  for (int i = 0; i < n; i++) {
    int t = targets[i];
    if (t == ignore) continue;
    int64_t b = (int64_t)i * vocab;
    float mx = -INFINITY;
    for (int v = 0; v < vocab; v++) if (src[(size_t)(b + v)] > mx) mx = src[(size_t)(b + v)];
    double se = 0;
    for (int v = 0; v < vocab; v++) se += exp((double)(src[(size_t)(b + v)] - mx));
    row_loss[(size_t)i] = ((double)mx + log(se)) - (double)src[(size_t)(b + t)];
  }
  double total = 0;
  int count = 0;
  for (int i = 0; i < n; i++) {
    if (targets[i] == ignore) continue;
    total += row_loss[(size_t)i];
    count++;
  }
  float loss = count > 0 ? (float)(total / count) : 0.0f;
  pai_tensor r;
  TRY(alloc(c, 0, nullptr, logits->dtype, &r));
  buf(r)[0] = loss;
  *out = r;
  return PAI_OK;
}

// CpuComputeBackend.CrossEntropyGrad (CpuComputeBackend.cs:477-500).
ORC_API pai_status oracle_cross_entropy_grad(pai_ctx* c, const pai_tensor* logits, const int32_t* targets, int64_t nt,
                                            int32_t ignore, pai_tensor* out) {
  CHECK_CTX(c);
  TRY(check_desc(c, logits, "logits"));
  if (logits->rank != 2) return fail(PAI_ERR_ARGUMENT, "CrossEntropyGrad: logits must be [N, vocab]");
  int n = logits->dims[0], vocab = logits->dims[1];
  if (nt < n) return fail(PAI_ERR_ARGUMENT, "targets (%lld) must have one entry per logits row (%d).", (long long)nt, n);
  auto src = materialize(*logits);
  int count = 0;
  for (int i = 0; i < n; i++) if (targets[i] != ignore) count++;
  for (int i = 0; i < n; i++) {
    int t = targets[i];
    if (t != ignore && (t < 0 || t >= vocab))
      return fail(PAI_ERR_OUT_OF_RANGE, "target out of range [0,%d). (Parameter 'targets') Actual value was %d.", vocab, t);
  }
  float inv_count = count > 0 ? 1.0f / (float)count : 0.0f;
  int32_t od[2] = {n, vocab};
  pai_tensor r;
  TRY(alloc(c, 2, od, logits->dtype, &r));
  float* dst = buf(r);
#pragma omp parallel for num_threads(g_threads) schedule(static) if ((int64_t)n * vocab > 65536)
  for (int i = 0; i < n; i++) {
    int t = targets[i];
    if (t == ignore) continue;
    int64_t b = (int64_t)i * vocab;
    float mx = -INFINITY;
    for (int v = 0; v < vocab; v++) {
      float x = src[(size_t)(b + v)];
      mx = (std::isnan(mx) || std::isnan(x)) ? NAN : (x > mx ? x : mx);  // MathF.Max
    }
    float se = 0.0f;
    for (int v = 0; v < vocab; v++) se += expf(src[(size_t)(b + v)] - mx);
    float inv = 1.0f / se;
    for (int v = 0; v < vocab; v++) dst[b + v] = expf(src[(size_t)(b + v)] - mx) * inv * inv_count;
    dst[b + t] -= inv_count;
  }
  *out = r;
  return PAI_OK;
}

// CpuComputeBackend.Cat (CpuComputeBackend.cs:509-540).
ORC_API pai_status oracle_cat(pai_ctx* c, const pai_tensor* a, const pai_tensor* b, int32_t axis, pai_tensor* out) {
  CHECK_CTX(c);
  TRY(check_desc(c, a, "a"));
  TRY(check_desc(c, b, "b"));
  int rank = a->rank;
  if (b->rank != rank) return fail(PAI_ERR_ARGUMENT, "Cat rank mismatch: %s vs %s.", shape_str(*a).c_str(), shape_str(*b).c_str());
  int ax = norm_axis(axis, rank);
  if (ax < 0 || ax >= rank) return fail(PAI_ERR_OUT_OF_RANGE, "Axis out of range for shape %s.", shape_str(*a).c_str());
  for (int i = 0; i < rank; i++)
    if (i != ax && a->dims[i] != b->dims[i])
      return fail(PAI_ERR_ARGUMENT, "Cat: dimensions must match except on axis %d: %s vs %s.", ax, shape_str(*a).c_str(), shape_str(*b).c_str());
  int64_t outer = 1, inner = 1;
  for (int i = 0; i < ax; i++) outer *= a->dims[i];
  for (int i = ax + 1; i < rank; i++) inner *= a->dims[i];
  int64_t la = a->dims[ax], lb = b->dims[ax], lt = la + lb;
  auto sa = materialize(*a);
  auto sb = materialize(*b);
  int32_t od[PAI_MAX_RANK];
  for (int i = 0; i < rank; i++) od[i] = a->dims[i];
  od[ax] = (int32_t)lt;
  pai_tensor r;
  TRY(alloc(c, rank, od, a->dtype, &r));
  float* dst = buf(r);
  for (int64_t o = 0; o < outer; o++) {
    if (la * inner != 0) memcpy(dst + o * lt * inner, sa.data() + o * la * inner, (size_t)(la * inner) * 4);
    if (lb * inner != 0) memcpy(dst + o * lt * inner + la * inner, sb.data() + o * lb * inner, (size_t)(lb * inner) * 4);
  }
  *out = r;
  return PAI_OK;
}


// ---------------------------------------------------------------- checkpoints (ProjectAI.Formats/Checkpoint.cs)
// The same entry points as the CUDA library's, synchronous: Checkpoint.Save (Checkpoint.cs:23-57) writes the file
// before returning (oracle_ckpt_wait has nothing to join), Checkpoint.Load (:63-110) reads every tensor into a host
// block of the current scope with the reader's checks. They let the host trainer's checkpoint flows run on the CPU.

ORC_API pai_status oracle_ckpt_save(pai_ctx* c, const char* path, int32_t step, const char* metadata, int64_t meta_len,
                                    const char* names, int64_t names_len, const pai_tensor* tensors, int32_t n) {
  CHECK_CTX(c);
  if (!path || n < 0 || meta_len < 0 || (n > 0 && (!tensors || !names))) return fail(PAI_ERR_ARGUMENT, "SaveCheckpoint: bad arguments");
  std::vector<std::string> nm;
  for (int64_t i = 0; i < names_len && (int)nm.size() < n;) {
    size_t len = strnlen(names + i, (size_t)(names_len - i));
    nm.emplace_back(names + i, len);
    i += (int64_t)len + 1;
  }
  if ((int)nm.size() != n) return fail(PAI_ERR_ARGUMENT, "SaveCheckpoint: %d names for %d tensors", (int)nm.size(), n);
  for (int i = 0; i < n; i++) {
    TRY(check_desc(c, &tensors[i], "tensor"));
    if (numel(tensors[i]) > 2147483647LL)
      return fail(PAI_ERR_UNSUPPORTED, "tensor '%s' has %lld elements, exceeding this format's 2^31 limit.", nm[(size_t)i].c_str(),
                  (long long)numel(tensors[i]));
  }
  FILE* f = fopen(path, "wb");
  if (!f) return fail(PAI_ERR_IO, "could not create '%s': %s", path, strerror(errno));
  bool ok = fwrite("PAICKPT2", 1, 8, f) == 8;
  auto w32 = [&](int32_t v) { ok = ok && fwrite(&v, 4, 1, f) == 1; };
  w32(step);
  w32((int32_t)meta_len);
  if (meta_len) ok = ok && fwrite(metadata, 1, (size_t)meta_len, f) == (size_t)meta_len;
  w32(n);
  for (int i = 0; i < n && ok; i++) {
    const pai_tensor& t = tensors[i];
    const std::string& name = nm[(size_t)i];
    w32((int32_t)name.size());
    if (!name.empty()) ok = ok && fwrite(name.data(), 1, name.size(), f) == name.size();
    w32(t.rank);
    for (int d = 0; d < t.rank; d++) w32(t.dims[d]);
    int64_t bytes = numel(t) * 4;
    ok = ok && fwrite(&bytes, 8, 1, f) == 1;
    auto dense = materialize(t);  // the view's logical elements in row-major order (ToHost)
    if (dense.size()) ok = ok && fwrite(dense.data(), 4, dense.size(), f) == dense.size();
  }
  if (fclose(f) != 0) ok = false;
  if (!ok) return fail(PAI_ERR_IO, "writing '%s' failed", path);
  return PAI_OK;
}

ORC_API pai_status oracle_ckpt_wait(pai_ctx* c) { CHECK_CTX(c); return PAI_OK; }

ORC_API pai_status oracle_ckpt_load(pai_ctx* c, const char* path, int32_t header_only, int32_t* step, int64_t* meta_len,
                                    int32_t* n_tensors) {
  CHECK_CTX(c);
  if (!path) return fail(PAI_ERR_ARGUMENT, "LoadCheckpoint: bad arguments");
  c->ck_meta.clear();
  c->ck_names.clear();
  c->ck_tensors.clear();
  FILE* f = fopen(path, "rb");
  if (!f) return fail(PAI_ERR_IO, "could not open '%s': %s", path, strerror(errno));
  struct Closer { FILE* f; ~Closer() { fclose(f); } } closer{f};
  auto exact = [&](void* dst, size_t n, const char* what) -> pai_status {
    size_t got = n ? fread(dst, 1, n, f) : 0;
    if (got != n)
      return fail(PAI_ERR_INVALID_DATA, "'%s' is truncated reading %s (expected %zu bytes, got %zu).", path, what, n, got);
    return PAI_OK;
  };
  char magic[8];
  if (fread(magic, 1, 8, f) != 8 || memcmp(magic, "PAICKPT2", 8) != 0)
    return fail(PAI_ERR_INVALID_DATA, "'%s' is not a ProjectAI checkpoint (bad magic).", path);
  int32_t stp = 0, mlen = 0, count = 0;
  TRY(exact(&stp, 4, "the step"));
  TRY(exact(&mlen, 4, "the metadata length"));
  if (mlen < 0 || mlen > (1 << 24)) return fail(PAI_ERR_INVALID_DATA, "'%s' has a bad metadata length (%d).", path, mlen);
  std::string meta((size_t)mlen, '\0');
  TRY(exact(mlen ? &meta[0] : nullptr, (size_t)mlen, "metadata"));
  if (step) *step = stp;
  if (meta_len) *meta_len = mlen;
  if (n_tensors) *n_tensors = 0;
  c->ck_meta = meta;
  if (header_only) return PAI_OK;
  TRY(exact(&count, 4, "the tensor count"));
  if (count < 0) return fail(PAI_ERR_INVALID_DATA, "'%s' has a negative tensor count (%d).", path, count);
  for (int32_t i = 0; i < count; i++) {
    int32_t nlen = 0, rank = 0;
    TRY(exact(&nlen, 4, "a tensor name length"));
    if (nlen < 0 || nlen > (1 << 20)) return fail(PAI_ERR_INVALID_DATA, "'%s' tensor %d: bad name length %d.", path, i, nlen);
    std::string name((size_t)nlen, '\0');
    std::string what = "tensor " + std::to_string(i) + " name";
    TRY(exact(nlen ? &name[0] : nullptr, (size_t)nlen, what.c_str()));
    TRY(exact(&rank, 4, "a tensor rank"));
    if (rank < 0 || rank > PAI_MAX_RANK) return fail(PAI_ERR_INVALID_DATA, "checkpoint tensor '%s' has invalid rank %d.", name.c_str(), rank);
    int32_t dims[PAI_MAX_RANK] = {};
    int64_t expected = 4;
    for (int d = 0; d < rank; d++) {
      TRY(exact(&dims[d], 4, "a tensor dimension"));
      if (dims[d] < 0) return fail(PAI_ERR_INVALID_DATA, "checkpoint tensor '%s' has a negative dimension %d.", name.c_str(), dims[d]);
      expected *= dims[d];
    }
    int64_t blen = 0;
    TRY(exact(&blen, 8, "a payload length"));
    if (blen != expected || blen > 2147483647LL)
      return fail(PAI_ERR_INVALID_DATA, "checkpoint tensor '%s': payload length %lld != dims product × 4 (%lld).", name.c_str(),
                  (long long)blen, (long long)expected);
    pai_tensor t;
    TRY(alloc(c, rank, dims, PAI_F32, &t));
    what = "tensor '" + name + "' payload";
    TRY(exact(t.base, (size_t)blen, what.c_str()));
    c->ck_names.push_back(name);
    c->ck_tensors.push_back(t);
  }
  if (n_tensors) *n_tensors = count;
  return PAI_OK;
}

ORC_API pai_status oracle_ckpt_meta(pai_ctx* c, char* b, int64_t cap) {
  CHECK_CTX(c);
  if ((int64_t)c->ck_meta.size() > cap || (!b && !c->ck_meta.empty())) return fail(PAI_ERR_ARGUMENT, "metadata buffer too small");
  if (!c->ck_meta.empty()) memcpy(b, c->ck_meta.data(), c->ck_meta.size());
  return PAI_OK;
}

ORC_API pai_status oracle_ckpt_tensor(pai_ctx* c, int32_t index, char* name, int64_t name_cap, int64_t* name_len, pai_tensor* out) {
  CHECK_CTX(c);
  if (index < 0 || index >= (int32_t)c->ck_tensors.size())
    return fail(PAI_ERR_OUT_OF_RANGE, "checkpoint tensor index %d out of range [0, %zu)", index, c->ck_tensors.size());
  const std::string& n = c->ck_names[(size_t)index];
  if (name_len) *name_len = (int64_t)n.size();
  if (name) {
    if (name_cap < (int64_t)n.size()) return fail(PAI_ERR_ARGUMENT, "name needs %zu bytes", n.size());
    if (!n.empty()) memcpy(name, n.data(), n.size());
  }
  if (out) *out = c->ck_tensors[(size_t)index];
  return PAI_OK;
}

ORC_API pai_status oracle_ckpt_close(pai_ctx* c) {
  CHECK_CTX(c);
  c->ck_names.clear();
  c->ck_tensors.clear();
  return PAI_OK;
}


// ---------------------------------------------------------------- packed datasets (ProjectAI.Training/PackedBinDataset.cs)
// PackedBinDataset.Open's checks on the shard (PackedBinDataset.cs:62-83) and NextBatch (Training.cs:122-141) over
// GetSequence (:96-117), on the host: inputs ids[:, :-1] and targets ids[:, 1:] of each drawn block as F32 ids.

ORC_API pai_status oracle_dataset_open(pai_ctx* c, const char* path, int32_t elem, int32_t seq, int64_t blocks) {
  CHECK_CTX(c);
  if (!path) return fail(PAI_ERR_ARGUMENT, "OpenDataset: bad arguments");
  if (elem != 2 && elem != 4) return fail(PAI_ERR_INVALID_DATA, "unsupported dataset dtype (%d-byte ids).", elem);
  if (seq < 1) return fail(PAI_ERR_INVALID_DATA, "manifest SequenceLength must be >= 1; got %d.", seq);
  if (blocks < 1) return fail(PAI_ERR_INVALID_DATA, "manifest BlockCount must be >= 1; got %lld.", (long long)blocks);
  if (blocks > 2147483647LL)
    return fail(PAI_ERR_INVALID_DATA, "manifest BlockCount %lld exceeds the dataset's int32 count.", (long long)blocks);
  FILE* f = fopen(path, "rb");
  if (!f) return fail(PAI_ERR_IO, "dataset shard '%s' (from manifest) not found: %s", path, strerror(errno));
  struct Closer { FILE* f; ~Closer() { fclose(f); } } closer{f};
  const int64_t needed = blocks * (int64_t)(seq + 1) * elem;
  std::vector<uint8_t> bytes((size_t)needed);
  size_t got = fread(bytes.data(), 1, (size_t)needed, f);
  if ((int64_t)got < needed) {
    fseek(f, 0, SEEK_END);
    return fail(PAI_ERR_INVALID_DATA, "dataset shard '%s' is %lld bytes but the manifest needs %lld for %lld blocks of %d %s ids.",
                path, (long long)ftell(f), (long long)needed, (long long)blocks, seq + 1, elem == 2 ? "u16" : "u32");
  }
  c->ds_bytes.swap(bytes);
  c->ds_elem = elem;
  c->ds_seq = seq;
  c->ds_blocks = blocks;
  return PAI_OK;
}

ORC_API pai_status oracle_dataset_batch(pai_ctx* c, const int64_t* indices, int32_t count, pai_tensor* inputs, pai_tensor* targets) {
  CHECK_CTX(c);
  if (c->ds_blocks == 0) return fail(PAI_ERR_INVALID_OP, "no dataset is open");
  if (count < 1 || !indices || !inputs || !targets) return fail(PAI_ERR_ARGUMENT, "NextBatch: bad arguments");
  const int seq = c->ds_seq, blk = seq + 1;
  for (int32_t r = 0; r < count; r++)
    if (indices[r] < 0 || indices[r] >= c->ds_blocks)
      return fail(PAI_ERR_OUT_OF_RANGE, "index %lld: valid range is [0, %lld).", (long long)indices[r], (long long)c->ds_blocks);
  std::vector<float> ids((size_t)count * blk);
  for (int32_t r = 0; r < count; r++) {
    const uint8_t* b = c->ds_bytes.data() + (size_t)indices[r] * blk * c->ds_elem;
    for (int t = 0; t < blk; t++) {
      uint32_t v;
      if (c->ds_elem == 2) {
        uint16_t h;
        memcpy(&h, b + (size_t)t * 2, 2);
        v = h;
      } else {
        memcpy(&v, b + (size_t)t * 4, 4);
        if (v > 2147483647u)  // GetSequence's checked((int)id)
          return fail(PAI_ERR_OUT_OF_RANGE, "id %u in block %lld exceeds the int32 range.", v, (long long)indices[r]);
      }
      ids[(size_t)r * blk + t] = (float)(int32_t)v;
    }
  }
  int32_t dims[2] = {count, seq};
  pai_tensor in, tg;
  TRY(alloc(c, 2, dims, PAI_F32, &in));
  TRY(alloc(c, 2, dims, PAI_F32, &tg));
  for (int32_t r = 0; r < count; r++)
    for (int t = 0; t < seq; t++) {
      buf(in)[(size_t)r * seq + t] = ids[(size_t)r * blk + t];
      buf(tg)[(size_t)r * seq + t] = ids[(size_t)r * blk + t + 1];
    }
  *inputs = in;
  *targets = tg;
  return PAI_OK;
}

ORC_API pai_status oracle_dataset_close(pai_ctx* c) {
  CHECK_CTX(c);
  std::vector<uint8_t>().swap(c->ds_bytes);
  c->ds_elem = c->ds_seq = 0;
  c->ds_blocks = 0;
  return PAI_OK;
}
