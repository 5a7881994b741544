// Single-axis reductions and softmax over a [outer, len, inner] decomposition of the (densified) input.
// Contract: IComputeBackend.cs:37-46; semantics CpuComputeBackend.cs:248-301 (Sum/Mean/Max, MathF.Max propagates
// NaN) and :322-358 (max-subtracted softmax). Sums run as tree reductions, so they differ from the oracle's
// sequential order by rounding only.
#include "common.cuh"

namespace pai {

enum RedKind { kRSum = 0, kRMean = 1, kRMax = 2 };

__device__ __forceinline__ float nanmax(float a, float b) {
  if (a != a || b != b) return __int_as_float(0x7fc00000);
  return a > b ? a : b;
}

template <int K>
__device__ __forceinline__ float red_combine(float a, float b) {
  return K == kRMax ? nanmax(a, b) : a + b;
}

template <int K>
__device__ __forceinline__ float warp_reduce(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = red_combine<K>(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Reduce contiguous rows (inner == 1): one block per row.
template <int K>
__global__ void k_reduce_rows(const float* __restrict__ x, float* __restrict__ o, int64_t rows, int len) {
  __shared__ float sm[32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* p = x + r * len;
    float acc = K == kRMax ? -INFINITY : 0.0f;
    for (int i = threadIdx.x; i < len; i += blockDim.x) acc = red_combine<K>(acc, p[i]);
    acc = warp_reduce<K>(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
      int nw = blockDim.x >> 5;
      float v = threadIdx.x < nw ? sm[threadIdx.x] : (K == kRMax ? -INFINITY : 0.0f);
      v = warp_reduce<K>(v);
      if (threadIdx.x == 0) o[r] = K == kRMean ? v / (float)len : v;
    }
    __syncthreads();
  }
}

// Reduce a middle axis (inner > 1): block (32 columns) x (8 row groups), shared-memory combine.
template <int K>
__global__ void k_reduce_cols(const float* __restrict__ x, float* __restrict__ o, int64_t outer, int len, int64_t inner) {
  __shared__ float sm[8][33];
  int64_t c = blockIdx.x * 32ll + threadIdx.x;
  for (int64_t ob = blockIdx.y; ob < outer; ob += gridDim.y) {
    float acc = K == kRMax ? -INFINITY : 0.0f;
    if (c < inner) {
      const float* p = x + ob * (int64_t)len * inner + c;
      for (int t = threadIdx.y; t < len; t += 8) acc = red_combine<K>(acc, p[(int64_t)t * inner]);
    }
    sm[threadIdx.y][threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.y == 0 && c < inner) {
      float v = sm[0][threadIdx.x];
      for (int j = 1; j < 8; j++) v = red_combine<K>(v, sm[j][threadIdx.x]);
      o[ob * inner + c] = K == kRMean ? v / (float)len : v;
    }
    __syncthreads();
  }
}

// Short middle axis (len <= 64, e.g. the batch fold of a broadcast weight gradient): one thread per output column,
// reading the axis sequentially — every load is coalesced across the warp.
template <int K>
__global__ void k_reduce_cols_short(const float* __restrict__ x, float* __restrict__ o, int64_t outer, int len, int64_t inner) {
  int64_t total = outer * inner;
  for (int64_t id = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; id < total; id += (int64_t)gridDim.x * blockDim.x) {
    int64_t ob = id / inner, c = id - ob * inner;
    const float* p = x + ob * (int64_t)len * inner + c;
    float acc = K == kRMax ? -INFINITY : 0.0f;
    for (int t = 0; t < len; t++) acc = red_combine<K>(acc, p[(int64_t)t * inner]);
    o[id] = K == kRMean ? acc / (float)len : acc;
  }
}

template <int K>
static pai_status reduce(pai_ctx* ctx, const pai_tensor* x, int axis, int keep, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_TRY(check_view(ctx, x, "x"));
  int rank = x->rank;
  if (rank == 0) return set_error(PAI_ERR_ARGUMENT, "Cannot reduce a scalar tensor.");
  int ax = norm_axis(axis, rank);
  if (ax < 0 || ax >= rank)
    return set_error(PAI_ERR_OUT_OF_RANGE, "Axis out of range for shape %s. (Parameter 'axis') Actual value was %d.",
                     shape_str(*x).c_str(), axis);
  int64_t outer = 1, inner = 1;
  for (int i = 0; i < ax; i++) outer *= x->dims[i];
  int len = x->dims[ax];
  for (int i = ax + 1; i < rank; i++) inner *= x->dims[i];
  int32_t od[PAI_MAX_RANK];
  int orank = 0;
  for (int i = 0; i < rank; i++) {
    if (i == ax) { if (keep) od[orank++] = 1; }
    else od[orank++] = x->dims[i];
  }
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, orank, od, x->dtype, false, &r));
  int64_t nout = outer * inner;
  if (nout > 0) {
    if (len == 0) {
      // Empty axis: sum/mean of nothing is 0 (mean 0/0 = NaN as in the oracle), max is -inf.
      float fill = K == kRMax ? -INFINITY : (K == kRMean ? NAN : 0.0f);
      std::vector<float> h((size_t)nout, fill);
      PAI_CUDA(cudaMemcpyAsync(fptr(r), h.data(), (size_t)nout * 4, cudaMemcpyHostToDevice, ctx->stream));
      PAI_CUDA(cudaStreamSynchronize(ctx->stream));
    } else {
      const float* src;
      Scratch hold;
      PAI_TRY(dense_input(ctx, *x, &src, &hold));
      if (inner == 1) {
        int threads = len >= 1024 ? 512 : (len >= 256 ? 256 : 128);
        int64_t blocks = outer < (int64_t)ctx->sm_count * 16 ? outer : (int64_t)ctx->sm_count * 16;
        k_reduce_rows<K><<<(int)blocks, threads, 0, ctx->stream>>>(src, fptr(r), outer, len);
      } else if (len <= 64 || outer * inner >= (int64_t)ctx->sm_count * 2048) {
        k_reduce_cols_short<K><<<grid_for(ctx, outer * inner, 256), 256, 0, ctx->stream>>>(src, fptr(r), outer, len, inner);
      } else {
        dim3 grid((unsigned)((inner + 31) / 32), (unsigned)(outer < 65535 ? outer : 65535));
        k_reduce_cols<K><<<grid, dim3(32, 8), 0, ctx->stream>>>(src, fptr(r), outer, len, inner);
      }
      PAI_LAUNCH_CHECK("reduce");
    }
  }
  *out = r;
  return PAI_OK;
}

// ---------------------------------------------------------------- softmax
// Contiguous axis: one block per row, three passes (max, sum of exp, normalise) over L1/L2-resident data.
__global__ void k_softmax_rows(const float* __restrict__ x, float* __restrict__ o, int64_t rows, int len) {
  __shared__ float sm[32];
  __shared__ float bc;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* p = x + r * len;
    float* q = o + r * len;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < len; i += blockDim.x) m = fmaxf(m, p[i]);
    m = warp_reduce<kRMax>(m);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : -INFINITY;
      v = warp_reduce<kRMax>(v);
      if (threadIdx.x == 0) bc = v;
    }
    __syncthreads();
    m = bc;
    __syncthreads();
    float s = 0.0f;
    for (int i = threadIdx.x; i < len; i += blockDim.x) {
      float e = expf(p[i] - m);
      q[i] = e;
      s += e;
    }
    s = warp_reduce<kRSum>(s);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0.0f;
      v = warp_reduce<kRSum>(v);
      if (threadIdx.x == 0) bc = v;
    }
    __syncthreads();
    float inv = 1.0f / bc;
    for (int i = threadIdx.x; i < len; i += blockDim.x) q[i] = q[i] * inv;
    __syncthreads();
  }
}

// Strided axis: one thread per (outer, inner) column.
__global__ void k_softmax_cols(const float* __restrict__ x, float* __restrict__ o, int64_t outer, int len, int64_t inner) {
  int64_t total = outer * inner;
  for (int64_t id = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; id < total; id += (int64_t)gridDim.x * blockDim.x) {
    int64_t ob = id / inner, c = id % inner;
    const float* p = x + ob * (int64_t)len * inner + c;
    float* q = o + ob * (int64_t)len * inner + c;
    float m = -INFINITY;
    for (int t = 0; t < len; t++) m = fmaxf(m, p[(int64_t)t * inner]);
    float s = 0.0f;
    for (int t = 0; t < len; t++) {
      float e = expf(p[(int64_t)t * inner] - m);
      q[(int64_t)t * inner] = e;
      s += e;
    }
    float inv = 1.0f / s;
    for (int t = 0; t < len; t++) q[(int64_t)t * inner] *= inv;
  }
}

}  // namespace pai

// ---------------------------------------------------------------- row argmax (greedy decoding)
// ArgMax of Sampling.cs:15-31 per row: NaN entries are skipped, ties resolve to the lowest index, and a row with no
// number gives index 0. Each thread scans its entries in index order keeping the first maximum; the block then keeps
// the larger value and, between equal values, the lower index, which is the sequential scan's answer.
__device__ __forceinline__ void argmax_keep(float v2, int i2, float& v1, int& i1) {
  if (i2 >= 0 && (i1 < 0 || v2 > v1 || (v2 == v1 && i2 < i1))) { v1 = v2; i1 = i2; }
}

__global__ void __launch_bounds__(256) k_argmax_rows(const float* __restrict__ x, int64_t row_stride, int n, int vec,
                                                     float* __restrict__ out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  const float* p = x + (int64_t)blockIdx.x * row_stride;
  float bv = -INFINITY;
  int bi = -1;
  if (vec) {
    for (int i4 = threadIdx.x; i4 < (n >> 2); i4 += blockDim.x) {
      float4 q = reinterpret_cast<const float4*>(p)[i4];
      float e[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; j++)
        if (!isnan(e[j]) && (bi < 0 || e[j] > bv)) { bv = e[j]; bi = 4 * i4 + j; }
    }
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float v = p[i];
      if (!isnan(v) && (bi < 0 || v > bv)) { bv = v; bi = i; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_keep(ov, oi, bv, bi);
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = sv[0];
    int i = si[0];
    for (int k = 1; k < nw; k++) argmax_keep(sv[k], si[k], v, i);
    out[blockIdx.x] = (float)(i < 0 ? 0 : i);
  }
}

using namespace pai;

PAI_API pai_status pai_argmax_rows(pai_ctx* ctx, const pai_tensor* x, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_TRY(check_view(ctx, x, "x"));
  if (x->rank < 1 || x->dims[x->rank - 1] < 1 || x->strides[x->rank - 1] != 1)
    return set_error(PAI_ERR_ARGUMENT, "ArgMaxRows: the last axis must be non-empty and unit-stride; got %s",
                     shape_str(*x).c_str());
  const int n = x->dims[x->rank - 1];
  // the leading axes must address the rows with one stride: consecutive non-unit axes nest, and the innermost one's
  // stride steps a row
  int64_t rows = 1, row_stride = n;
  int prev = -1;
  for (int i = 0; i < x->rank - 1; i++) {
    rows *= x->dims[i];
    if (x->dims[i] == 1) continue;
    if (prev >= 0 && x->strides[prev] != x->strides[i] * x->dims[i])
      return set_error(PAI_ERR_UNSUPPORTED, "ArgMaxRows: the leading axes of %s do not collapse to one row stride",
                       shape_str(*x).c_str());
    prev = i;
  }
  if (prev >= 0) row_stride = x->strides[prev];
  if (rows > INT32_MAX) return set_error(PAI_ERR_UNSUPPORTED, "ArgMaxRows: too many rows");
  int32_t od[1] = {(int32_t)rows};
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, 1, od, x->dtype, false, &r));
  if (rows > 0) {
    const float* base = fptr(*x);
    int vec = (n % 4 == 0) && (reinterpret_cast<uintptr_t>(base) % 16 == 0) && (row_stride % 4 == 0);
    k_argmax_rows<<<(unsigned)rows, 256, 0, ctx->stream>>>(base, row_stride, n, vec, fptr(r));
    PAI_LAUNCH_CHECK("argmax rows");
  }
  *out = r;
  return PAI_OK;
}

PAI_API pai_status pai_sum(pai_ctx* c, const pai_tensor* x, int32_t a, int32_t k, pai_tensor* o) { return reduce<kRSum>(c, x, a, k, o); }
PAI_API pai_status pai_mean(pai_ctx* c, const pai_tensor* x, int32_t a, int32_t k, pai_tensor* o) { return reduce<kRMean>(c, x, a, k, o); }
PAI_API pai_status pai_max(pai_ctx* c, const pai_tensor* x, int32_t a, int32_t k, pai_tensor* o) { return reduce<kRMax>(c, x, a, k, o); }

PAI_API pai_status pai_softmax(pai_ctx* ctx, const pai_tensor* x, int32_t axis, pai_tensor* out) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> g(ctx->mu);
  PAI_TRY(check_view(ctx, x, "x"));
  int rank = x->rank;
  if (rank == 0) return set_error(PAI_ERR_ARGUMENT, "Softmax requires rank >= 1.");
  int ax = norm_axis(axis, rank);
  if (ax < 0 || ax >= rank) return set_error(PAI_ERR_OUT_OF_RANGE, "Specified argument was out of the range of valid values. (Parameter 'axis')");
  int64_t outer = 1, inner = 1;
  for (int i = 0; i < ax; i++) outer *= x->dims[i];
  int len = x->dims[ax];
  for (int i = ax + 1; i < rank; i++) inner *= x->dims[i];
  pai_tensor r;
  PAI_TRY(alloc_tensor(ctx, rank, x->dims, x->dtype, false, &r));
  if (numel(r) > 0) {
    const float* src;
    Scratch hold;
    PAI_TRY(dense_input(ctx, *x, &src, &hold));
    if (inner == 1) {
      int threads = len >= 1024 ? 512 : (len >= 256 ? 256 : 128);
      int64_t blocks = outer < (int64_t)ctx->sm_count * 16 ? outer : (int64_t)ctx->sm_count * 16;
      k_softmax_rows<<<(int)blocks, threads, 0, ctx->stream>>>(src, fptr(r), outer, len);
    } else {
      k_softmax_cols<<<grid_for(ctx, outer * inner, 256), 256, 0, ctx->stream>>>(src, fptr(r), outer, len, inner);
    }
    PAI_LAUNCH_CHECK("softmax");
  }
  *out = r;
  return PAI_OK;
}
