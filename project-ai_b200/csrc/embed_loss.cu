// Embedding gather / scatter-add, cross-entropy over the vocabulary, and Cat.
// Semantics: CpuComputeBackend.cs:424-451 (Gather, ScatterAddRows: per-id rows summed in id order, so the
// result is bit-exact), :453-500 (CrossEntropy with double accumulation, CrossEntropyGrad in float), :509-540 (Cat).
// Ids and targets arrive as host int arrays (the contract's int[]); range checks run on the host before launch,
// raising ArgumentOutOfRange as the reference does.
#include <algorithm>
#include <numeric>
#include <vector>

#include "common.cuh"
#include "tc_common.cuh"

namespace pai {

__global__ void k_gather_rows(const float* __restrict__ table, const int32_t* __restrict__ ids, float* __restrict__ out,
                              int64_t n, int dim) {
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const float* src = table + (int64_t)ids[r] * dim;
    float* dst = out + r * dim;
    for (int j = threadIdx.x; j < dim; j += blockDim.x) dst[j] = src[j];
  }
}

// Gather with ids read from a device tensor (integral F32 values). An id outside [0, vocab) sets the device error flag
// and yields a zero row.
__global__ void k_gather_rows_dev(const float* __restrict__ table, const float* __restrict__ ids, float* __restrict__ out,
                                  int64_t n, int dim, int vocab, int* error_flag) {
  pdl_trigger();
  pdl_wait();
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    float f = ids[r];
    int id = (int)f;
    bool ok = f >= 0.0f && id < vocab && (float)id == f;
    if (!ok && threadIdx.x == 0) atomicExch(error_flag, 62);
    const float* src = table + (int64_t)(ok ? id : 0) * dim;
    float* dst = out + r * dim;
    for (int j = threadIdx.x; j < dim; j += blockDim.x) dst[j] = ok ? src[j] : 0.0f;
  }
}

// One block per distinct id: rows of that id summed in their original order, starting from zero.
__global__ void k_scatter_rows(const float* __restrict__ rows, const int32_t* __restrict__ uniq, const int32_t* __restrict__ start,
                               const int32_t* __restrict__ pos, float* __restrict__ out, int n_uniq, int dim) {
  for (int u = blockIdx.x; u < n_uniq; u += gridDim.x) {
    int id = uniq[u], s = start[u], e = start[u + 1];
    for (int j = threadIdx.x; j < dim; j += blockDim.x) {
      float acc = 0.0f;
      for (int k = s; k < e; k++) acc = __fadd_rn(acc, rows[(int64_t)pos[k] * dim + j]);
      out[(int64_t)id * dim + j] = acc;
    }
  }
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = -INFINITY;
#pragma unroll
  for (int i = 0; i < NT / 32; i++) r = fmaxf(r, sm[i]);
  __syncthreads();
  return r;
}

template <int NT>
__device__ __forceinline__ double block_sum_d(double v, double* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = 0.0;
#pragma unroll
  for (int i = 0; i < NT / 32; i++) r += sm[i];
  __syncthreads();
  return r;
}

template <int NT>
__device__ __forceinline__ float block_sum_f(float v, float* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / 32; i++) r += sm[i];
  __syncthreads();
  return r;
}

// Cross-entropy value per row (double log-sum-exp as CpuComputeBackend.cs:462-473), written to row_loss; ignored rows get 0.
template <int NT>
__global__ void k_ce_rows(const float* __restrict__ logits, const int32_t* __restrict__ targets, double* __restrict__ row_loss,
                          int n, int vocab, int ignore) {
  __shared__ float smf[NT / 32];
  __shared__ double smd[NT / 32];
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    int t = targets[r];
    if (t == ignore) {
      if (threadIdx.x == 0) row_loss[r] = 0.0;
      continue;
    }
    const float* p = logits + (int64_t)r * vocab;
    float m = -INFINITY;
    for (int v = threadIdx.x; v < vocab; v += NT) m = fmaxf(m, p[v]);
    m = block_max<NT>(m, smf);
    double se = 0.0;
    float sef = 0.0f;
    for (int v = threadIdx.x; v < vocab; v += NT) sef += expf(p[v] - m);
    se = block_sum_d<NT>((double)sef, smd);
    if (threadIdx.x == 0) row_loss[r] = ((double)m + log(se)) - (double)p[t];
  }
}

// Deterministic tree sum of the per-row losses into a float scalar mean.
__global__ void k_ce_total(const double* __restrict__ row_loss, int n, int count, float* __restrict__ out) {
  __shared__ double sm[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += row_loss[i];
  acc = block_sum_d<1024>(acc, sm);
  if (threadIdx.x == 0) out[0] = count > 0 ? (float)(acc / count) : 0.0f;
}

// (softmax − onehot)·inv_count·scale per row (CpuComputeBackend.cs:477-500). The row stays in registers: VPT values per
// thread, so the logits are read once and the gradient written once.
template <int NT, int VPT>
__global__ void k_ce_grad_reg(const float* __restrict__ logits, const int32_t* __restrict__ targets, float* __restrict__ grad,
                              double* __restrict__ row_loss, int n, int vocab, int ignore, float inv_count, float scale) {
  __shared__ float smf[NT / 32];
  __shared__ double smd[NT / 32];
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    int t = targets[r];
    float* g = grad + (int64_t)r * vocab;
    if (t == ignore) {
      for (int v = threadIdx.x; v < vocab; v += NT) g[v] = 0.0f;
      if (row_loss && threadIdx.x == 0) row_loss[r] = 0.0;
      continue;
    }
    const float* p = logits + (int64_t)r * vocab;
    float x[VPT];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; k++) {
      int v = threadIdx.x + k * NT;
      x[k] = v < vocab ? p[v] : -INFINITY;
      m = fmaxf(m, x[k]);
    }
    m = block_max<NT>(m, smf);
    float sef = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; k++) {
      int v = threadIdx.x + k * NT;
      x[k] = v < vocab ? expf(x[k] - m) : 0.0f;
      sef += x[k];
    }
    double se = block_sum_d<NT>((double)sef, smd);
    float inv = 1.0f / (float)se;
#pragma unroll
    for (int k = 0; k < VPT; k++) {
      int v = threadIdx.x + k * NT;
      if (v < vocab) {
        float gv = x[k] * inv * inv_count;
        if (v == t) gv -= inv_count;
        g[v] = gv * scale;
      }
    }
    if (row_loss && threadIdx.x == 0) row_loss[r] = ((double)m + log(se)) - (double)p[t];
  }
}

// Rows of up to NT·VPT logits whose byte length is a multiple of 16 (vocab % 4 == 0): the arithmetic of k_ce_grad_reg
// (each thread holds the same VPT values and the reductions run in the same order, so the results are bit-identical),
// with one CTA per SM walking its rows while the next row's logits stream into shared memory as one bulk copy. The
// HBM read of row i+gridDim.x then overlaps the exponentials and gradient stores of row i, where the register kernel
// (one CTA per SM: its registers hold a whole row) reads, computes and writes each row in turn. A copy that has not
// landed within the wait limit sets the device error flag (site 81) and the CTA stops.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT, 1)
    k_ce_grad_stream(const float* __restrict__ logits, const int32_t* __restrict__ targets, float* __restrict__ grad,
                     double* __restrict__ row_loss, int n, int vocab, int ignore, float inv_count, float scale,
                     int* __restrict__ error_flag) {
  extern __shared__ __align__(128) uint8_t ce_smem[];
  float* row = reinterpret_cast<float*>(ce_smem);
  __shared__ __align__(8) uint64_t bar;
  __shared__ float smf[NT / 32];
  __shared__ double smd[NT / 32];
  const uint32_t bytes = (uint32_t)vocab * 4u;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if ((int)blockIdx.x < n) {
      tc::mbar_expect_tx(&bar, bytes);
      tc::bulk_g2s(row, logits + (int64_t)blockIdx.x * vocab, bytes, &bar);
    }
  }
  __syncthreads();
  uint32_t parity = 0;
  for (int r = blockIdx.x; r < n; r += gridDim.x, parity ^= 1u) {
    // every thread waits on the barrier (acquiring the copy's writes); the CTA agrees on the outcome in one barrier
    if (!__syncthreads_and(tc::mbar_wait(&bar, parity) ? 1 : 0)) {
      if (threadIdx.x == 0) {
        atomicExch(error_flag, 81);
        tc::mbar_wait(&bar, parity);  // bounded: a late copy lands before the CTA's shared memory is released
      }
      return;
    }
    const int t = targets[r];
    float x[VPT];
#pragma unroll
    for (int k = 0; k < VPT; k++) {
      int v = threadIdx.x + k * NT;
      x[k] = v < vocab ? row[v] : -INFINITY;
    }
    float xt = 0.0f;
    if (threadIdx.x == 0 && t != ignore) xt = row[t];
    __syncthreads();  // every thread has its values: the buffer takes the next row
    if (threadIdx.x == 0 && r + (int)gridDim.x < n) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the reads above come before the copy's writes
      tc::mbar_expect_tx(&bar, bytes);
      tc::bulk_g2s(row, logits + (int64_t)(r + gridDim.x) * vocab, bytes, &bar);
    }
    float* g = grad + (int64_t)r * vocab;
    if (t == ignore) {
      for (int v = threadIdx.x; v < vocab; v += NT) g[v] = 0.0f;
      if (row_loss && threadIdx.x == 0) row_loss[r] = 0.0;
      continue;
    }
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; k++) m = fmaxf(m, x[k]);
    m = block_max<NT>(m, smf);
    float sef = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; k++) {
      int v = threadIdx.x + k * NT;
      x[k] = v < vocab ? expf(x[k] - m) : 0.0f;
      sef += x[k];
    }
    double se = block_sum_d<NT>((double)sef, smd);
    float inv = 1.0f / (float)se;
#pragma unroll
    for (int k = 0; k < VPT; k++) {
      int v = threadIdx.x + k * NT;
      if (v < vocab) {
        float gv = x[k] * inv * inv_count;
        if (v == t) gv -= inv_count;
        g[v] = gv * scale;
      }
    }
    if (row_loss && threadIdx.x == 0) row_loss[r] = ((double)m + log(se)) - (double)xt;
  }
}

// Any vocabulary size: three passes over the row.
template <int NT>
__global__ void k_ce_grad_loop(const float* __restrict__ logits, const int32_t* __restrict__ targets, float* __restrict__ grad,
                               double* __restrict__ row_loss, int n, int vocab, int ignore, float inv_count, float scale) {
  __shared__ float smf[NT / 32];
  __shared__ double smd[NT / 32];
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    int t = targets[r];
    float* g = grad + (int64_t)r * vocab;
    if (t == ignore) {
      for (int v = threadIdx.x; v < vocab; v += NT) g[v] = 0.0f;
      if (row_loss && threadIdx.x == 0) row_loss[r] = 0.0;
      continue;
    }
    const float* p = logits + (int64_t)r * vocab;
    float m = -INFINITY;
    for (int v = threadIdx.x; v < vocab; v += NT) m = fmaxf(m, p[v]);
    m = block_max<NT>(m, smf);
    float sef = 0.0f;
    for (int v = threadIdx.x; v < vocab; v += NT) sef += expf(p[v] - m);
    double se = block_sum_d<NT>((double)sef, smd);
    float inv = 1.0f / (float)se;
    for (int v = threadIdx.x; v < vocab; v += NT) {
      float gv = expf(p[v] - m) * inv * inv_count;
      if (v == t) gv -= inv_count;
      g[v] = gv * scale;
    }
    if (row_loss && threadIdx.x == 0) row_loss[r] = ((double)m + log(se)) - (double)p[t];
  }
}

static pai_status check_targets(const int32_t* targets, int64_t nt, int n, int vocab, int ignore, int* count) {
  if (nt < n) return set_error(PAI_ERR_ARGUMENT, "targets (%lld) must have one entry per logits row (%d).", (long long)nt, n);
  int c = 0;
  for (int i = 0; i < n; i++) {
    int t = targets[i];
    if (t == ignore) continue;
    if (t < 0 || t >= vocab)
      return set_error(PAI_ERR_OUT_OF_RANGE, "target out of range [0,%d). (Parameter 'targets') Actual value was %d.", vocab, t);
    c++;
  }
  *count = c;
  return PAI_OK;
}

static pai_status launch_ce_grad(pai_ctx* ctx, const float* lp, const int32_t* dt, float* grad, double* row_loss, int n,
                                 int vocab, int ignore, float inv_count, float scale) {
  int blocks = n < ctx->sm_count * 8 ? n : ctx->sm_count * 8;
  if (blocks < 1) return PAI_OK;
  // Rows up to 16K stay in registers with 1024 threads; up to 32K with 512 threads x 64 values (<= 128 regs).
  int vpt = (vocab + 1023) / 1024;
#define CE_REG(T, V) k_ce_grad_reg<T, V><<<blocks, T, 0, ctx->stream>>>(lp, dt, grad, row_loss, n, vocab, ignore, inv_count, scale)
  if (vpt <= 1) CE_REG(1024, 1);
  else if (vpt <= 2) CE_REG(1024, 2);
  else if (vpt <= 4) CE_REG(1024, 4);
  else if (vpt <= 8) CE_REG(1024, 8);
  else if (vpt <= 16) CE_REG(1024, 16);
  else if (vocab <= 32768) {
    if (vocab % 4 == 0 && (reinterpret_cast<uintptr_t>(lp) & 15) == 0) {
      // bulk copies start on 16-byte boundaries: every row does when the base does and rows are whole float4s
      const int smem = vocab * 4;
      PAI_CUDA(smem_limit(ctx, k_ce_grad_stream<512, 64>, smem));
      const int grid = n < ctx->sm_count ? n : ctx->sm_count;
      k_ce_grad_stream<512, 64><<<grid, 512, smem, ctx->stream>>>(lp, dt, grad, row_loss, n, vocab, ignore, inv_count,
                                                                   scale, ctx->d_error_flag);
    } else {
      CE_REG(512, 64);
    }
  } else k_ce_grad_loop<1024><<<blocks, 1024, 0, ctx->stream>>>(lp, dt, grad, row_loss, n, vocab, ignore, inv_count, scale);
#undef CE_REG
  PAI_LAUNCH_CHECK("cross_entropy_grad");
  return PAI_OK;
}

}  // namespace pai

using namespace pai;

PAI_API pai_status pai_gather(pai_ctx* ctx, const pai_tensor* table, const int32_t* ids, int64_t n, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, table, "table"));
  if (table->rank != 2) return set_error(PAI_ERR_ARGUMENT, "Gather: table must be [vocab, dim], got %s", shape_str(*table).c_str());
  int vocab = table->dims[0], dim = table->dims[1];
  for (int64_t i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= vocab)
      return set_error(PAI_ERR_OUT_OF_RANGE, "id out of range [0,%d). (Parameter 'ids') Actual value was %d.", vocab, ids[i]);
  int32_t od[2] = {(int32_t)n, dim};
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, 2, od, table->dtype, false, &r));
  if (n > 0 && dim > 0) {
    const float* tp;
    Scratch ht, hid;
    PAI_TRY(dense_input(ctx, *table, &tp, &ht));
    PAI_TRY(upload(ctx, ids, (size_t)n * 4, &hid));
    int blocks = n < ctx->sm_count * 16 ? (int)n : ctx->sm_count * 16;
    k_gather_rows<<<blocks, 256, 0, ctx->stream>>>(tp, static_cast<int32_t*>(hid.p), fptr(r), n, dim);
    PAI_LAUNCH_CHECK("gather");
  }
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_gather_dev(pai_ctx* ctx, const pai_tensor* table, const pai_tensor* ids, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, table, "table"));
  PAI_TRY(check_view(ctx, ids, "ids"));
  if (table->rank != 2) return set_error(PAI_ERR_ARGUMENT, "Gather: table must be [vocab, dim], got %s", shape_str(*table).c_str());
  if (ids->rank + 1 > PAI_MAX_RANK) return set_error(PAI_ERR_ARGUMENT, "Gather: ids rank too large");
  if (!is_dense(*ids)) return set_error(PAI_ERR_ARGUMENT, "Gather: ids must be a dense tensor");
  int vocab = table->dims[0], dim = table->dims[1];
  int32_t od[PAI_MAX_RANK];
  for (int i = 0; i < ids->rank; i++) od[i] = ids->dims[i];
  od[ids->rank] = dim;
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, ids->rank + 1, od, table->dtype, false, &r));
  int64_t n = numel(*ids);
  if (n > 0 && dim > 0) {
    const float* tp;
    Scratch ht;
    PAI_TRY(dense_input(ctx, *table, &tp, &ht));
    int blocks = n < ctx->sm_count * 16 ? (int)n : ctx->sm_count * 16;
    PAI_PDL_LAUNCH(launch_pdl(k_gather_rows_dev, dim3(blocks), dim3(256), 0, ctx->stream, tp,
                              static_cast<const float*>(fptr(*ids)), fptr(r), n, dim, vocab, ctx->d_error_flag),
                   "gather_dev");
  }
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_scatter_add_rows(pai_ctx* ctx, const pai_tensor* rows, const int32_t* ids, int64_t n, int32_t row_count,
                                        pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, rows, "rows"));
  if (rows->rank < 1) return set_error(PAI_ERR_ARGUMENT, "ScatterAddRows: rows must have rank >= 1");
  int dim = rows->dims[rows->rank - 1];
  if (numel(*rows) < n * dim) return set_error(PAI_ERR_ARGUMENT, "ScatterAddRows: %lld ids but fewer rows", (long long)n);
  for (int64_t i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= row_count)
      return set_error(PAI_ERR_OUT_OF_RANGE, "id out of range [0,%d). (Parameter 'ids') Actual value was %d.", row_count, ids[i]);
  int32_t od[2] = {row_count, dim};
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, 2, od, rows->dtype, true, &r));
  if (n > 0 && dim > 0) {
    // Host CSR: distinct ids and, per id, the row positions in their original order.
    std::vector<int32_t> order((size_t)n);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return ids[a] < ids[b]; });
    std::vector<int32_t> uniq, start;
    for (int64_t k = 0; k < n; k++) {
      if (k == 0 || ids[order[(size_t)k]] != ids[order[(size_t)k - 1]]) {
        uniq.push_back(ids[order[(size_t)k]]);
        start.push_back((int32_t)k);
      }
    }
    start.push_back((int32_t)n);
    std::vector<int32_t> packed;
    packed.reserve(uniq.size() * 2 + 1 + (size_t)n);
    packed.insert(packed.end(), uniq.begin(), uniq.end());
    packed.insert(packed.end(), start.begin(), start.end());
    packed.insert(packed.end(), order.begin(), order.end());
    const float* rp;
    Scratch hr, hp;
    PAI_TRY(dense_input(ctx, *rows, &rp, &hr));
    PAI_TRY(upload(ctx, packed.data(), packed.size() * 4, &hp));
    const int32_t* d = static_cast<const int32_t*>(hp.p);
    int nu = (int)uniq.size();
    int blocks = nu < ctx->sm_count * 16 ? nu : ctx->sm_count * 16;
    k_scatter_rows<<<blocks, 256, 0, ctx->stream>>>(rp, d, d + nu, d + 2 * nu + 1, fptr(r), nu, dim);
    PAI_LAUNCH_CHECK("scatter_add_rows");
  }
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_cross_entropy(pai_ctx* ctx, const pai_tensor* logits, const int32_t* targets, int64_t nt, int32_t ignore,
                                     pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, logits, "logits"));
  if (logits->rank != 2) return set_error(PAI_ERR_ARGUMENT, "CrossEntropy: logits must be [N, vocab], got %s", shape_str(*logits).c_str());
  int n = logits->dims[0], vocab = logits->dims[1], count = 0;
  PAI_TRY(check_targets(targets, nt, n, vocab, ignore, &count));
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, 0, nullptr, logits->dtype, true, &r));
  if (n > 0) {
    const float* lp;
    Scratch hl, ht, hloss;
    PAI_TRY(dense_input(ctx, *logits, &lp, &hl));
    PAI_TRY(upload(ctx, targets, (size_t)n * 4, &ht));
    PAI_TRY(scratch(ctx, (size_t)n * 8, &hloss));
    int blocks = n < ctx->sm_count * 8 ? n : ctx->sm_count * 8;
    k_ce_rows<512><<<blocks, 512, 0, ctx->stream>>>(lp, static_cast<int32_t*>(ht.p), static_cast<double*>(hloss.p), n, vocab, ignore);
    PAI_LAUNCH_CHECK("cross_entropy");
    k_ce_total<<<1, 1024, 0, ctx->stream>>>(static_cast<double*>(hloss.p), n, count, fptr(r));
    PAI_LAUNCH_CHECK("cross_entropy total");
  }
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_cross_entropy_grad(pai_ctx* ctx, const pai_tensor* logits, const int32_t* targets, int64_t nt,
                                          int32_t ignore, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, logits, "logits"));
  if (logits->rank != 2) return set_error(PAI_ERR_ARGUMENT, "CrossEntropyGrad: logits must be [N, vocab], got %s", shape_str(*logits).c_str());
  int n = logits->dims[0], vocab = logits->dims[1], count = 0;
  PAI_TRY(check_targets(targets, nt, n, vocab, ignore, &count));
  float inv_count = count > 0 ? 1.0f / (float)count : 0.0f;
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, 2, logits->dims, logits->dtype, false, &r));
  if (n > 0 && vocab > 0) {
    const float* lp;
    Scratch hl, ht;
    PAI_TRY(dense_input(ctx, *logits, &lp, &hl));
    PAI_TRY(upload(ctx, targets, (size_t)n * 4, &ht));
    PAI_TRY(launch_ce_grad(ctx, lp, static_cast<int32_t*>(ht.p), fptr(r), nullptr, n, vocab, ignore, inv_count, 1.0f));
  }
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_cross_entropy_fused(pai_ctx* ctx, const pai_tensor* logits, const int32_t* targets, int64_t nt,
                                           int32_t ignore, float grad_scale, pai_tensor* loss, pai_tensor* grad) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, logits, "logits"));
  if (logits->rank != 2) return set_error(PAI_ERR_ARGUMENT, "CrossEntropy: logits must be [N, vocab], got %s", shape_str(*logits).c_str());
  int n = logits->dims[0], vocab = logits->dims[1], count = 0;
  PAI_TRY(check_targets(targets, nt, n, vocab, ignore, &count));
  float inv_count = count > 0 ? 1.0f / (float)count : 0.0f;
  pai_tensor rl, rg;
  PAI_TRY(alloc_tensor(ctx, 0, nullptr, logits->dtype, true, &rl));
  PAI_TRY(alloc_tensor(ctx, 2, logits->dims, logits->dtype, false, &rg));
  if (n > 0 && vocab > 0) {
    const float* lp;
    Scratch hl, ht, hloss;
    PAI_TRY(dense_input(ctx, *logits, &lp, &hl));
    PAI_TRY(upload(ctx, targets, (size_t)n * 4, &ht));
    PAI_TRY(scratch(ctx, (size_t)n * 8, &hloss));
    PAI_TRY(launch_ce_grad(ctx, lp, static_cast<int32_t*>(ht.p), fptr(rg), static_cast<double*>(hloss.p), n, vocab, ignore,
                           inv_count, grad_scale));
    k_ce_total<<<1, 1024, 0, ctx->stream>>>(static_cast<double*>(hloss.p), n, count, fptr(rl));
    PAI_LAUNCH_CHECK("cross_entropy total");
  }
  *loss = rl;
  *grad = rg;
  return PAI_OK;
}

PAI_API pai_status pai_cat(pai_ctx* ctx, const pai_tensor* a, const pai_tensor* b, int32_t axis, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  PAI_TRY(check_view(ctx, a, "a"));
  PAI_TRY(check_view(ctx, b, "b"));
  int rank = a->rank;
  if (b->rank != rank) return set_error(PAI_ERR_ARGUMENT, "Cat rank mismatch: %s vs %s.", shape_str(*a).c_str(), shape_str(*b).c_str());
  int ax = norm_axis(axis, rank);
  if (ax < 0 || ax >= rank) return set_error(PAI_ERR_OUT_OF_RANGE, "Axis out of range for shape %s.", shape_str(*a).c_str());
  for (int i = 0; i < rank; i++)
    if (i != ax && a->dims[i] != b->dims[i])
      return set_error(PAI_ERR_ARGUMENT, "Cat: dimensions must match except on axis %d: %s vs %s.", ax, shape_str(*a).c_str(),
                       shape_str(*b).c_str());
  int32_t od[PAI_MAX_RANK];
  for (int i = 0; i < rank; i++) od[i] = a->dims[i];
  od[ax] = a->dims[ax] + b->dims[ax];
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, rank, od, a->dtype, false, &r));
  // Each operand is copied into its slice of the result: a view of r with the operand's shape.
  for (int part = 0; part < 2; part++) {
    const pai_tensor* src = part == 0 ? a : b;
    if (numel(*src) == 0) continue;
    pai_tensor dst = r;
    dst.dims[ax] = src->dims[ax];
    dst.offset = part == 0 ? 0 : (int64_t)a->dims[ax] * r.strides[ax];
    PAI_TRY(pai_copy(ctx, src, &dst));
  }
  *out = r;
  return PAI_OK;
}
