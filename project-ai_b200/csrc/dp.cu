// Data parallelism: one process per GPU, gradient buckets summed with NCCL all-reduce on a dedicated stream so the
// exchange of one transformer block's gradients overlaps the backward of the blocks before it.
// The reference is single-device; this is the data-parallel extension of its trainer.
// The communicator is created non-blocking. Every NCCL call is polled under a host deadline (ncclInProgress), and
// pai_allreduce_wait polls the completion of the enqueued all-reduces under the same deadline together with
// ncclCommGetAsyncError. A peer that died before or during an exchange therefore ends in PAI_ERR_NCCL or
// PAI_ERR_TIMEOUT: the communicator is aborted, which ends its kernels, so the compute stream is not left waiting
// on a collective that cannot finish.
#include <nccl.h>

#include <chrono>
#include <thread>

#include "common.cuh"

namespace pai {

// Exposed exchange time: per step, the device time from the end of the backward on the compute stream (recorded as
// pai_allreduce_wait is called) to the end of the last all-reduce on the communication stream; zero when the exchange
// finished first. A ring of event pairs is read back lazily by pai_dp_stats once both events of a pair completed.
constexpr int kStatRing = 64;

struct NcclState {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  int timeout_ms = 60000;
  cudaEvent_t ready = nullptr;  // compute stream -> comm stream
  cudaEvent_t done = nullptr;   // comm stream -> compute stream
  bool pending = false;
  cudaEvent_t bwd_end[kStatRing] = {};  // timing events on the compute stream
  cudaEvent_t ar_end[kStatRing] = {};   // timing events on the comm stream
  int64_t recorded = 0, read = 0;       // pairs recorded / pairs accounted
  double exposed_ms = 0.0;
  int64_t exposed_steps = 0;
};

static void abort_comm(NcclState* s) {
  if (s->comm) {
    ncclCommAbort(s->comm);
    s->comm = nullptr;
  }
}

static pai_status nccl_wait(NcclState* s, ncclResult_t r, const char* what) {
  auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(s->timeout_ms);
  while (r == ncclInProgress) {
    if (std::chrono::steady_clock::now() > deadline) {
      abort_comm(s);
      return set_error(PAI_ERR_TIMEOUT, "NCCL %s did not complete within %d ms; communicator aborted", what, s->timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    ncclCommGetAsyncError(s->comm, &r);
  }
  if (r != ncclSuccess) {
    abort_comm(s);
    return set_error(PAI_ERR_NCCL, "NCCL %s failed: %s", what, ncclGetErrorString(r));
  }
  return PAI_OK;
}

// Host-side wait for `ev` (recorded on the comm stream after the last all-reduce) under the deadline, checking the
// communicator's asynchronous error between polls.
static pai_status wait_done(NcclState* s, cudaEvent_t ev) {
  auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(s->timeout_ms);
  for (;;) {
    cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return PAI_OK;
    if (q != cudaErrorNotReady) {
      abort_comm(s);
      return set_error(PAI_ERR_CUDA, "all-reduce completion: %s", cudaGetErrorString(q));
    }
    ncclResult_t r = ncclSuccess;
    if (s->comm) ncclCommGetAsyncError(s->comm, &r);
    if (r != ncclSuccess && r != ncclInProgress) {
      abort_comm(s);
      return set_error(PAI_ERR_NCCL, "NCCL all-reduce failed: %s; communicator aborted", ncclGetErrorString(r));
    }
    if (std::chrono::steady_clock::now() > deadline) {
      abort_comm(s);
      return set_error(PAI_ERR_TIMEOUT, "NCCL all-reduce did not complete within %d ms (a peer left?); communicator aborted",
                       s->timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// Accounts every recorded (backward end, all-reduce end) pair whose events have completed.
static void read_stats(NcclState* s) {
  while (s->read < s->recorded) {
    const int i = (int)(s->read % kStatRing);
    if (cudaEventQuery(s->bwd_end[i]) != cudaSuccess || cudaEventQuery(s->ar_end[i]) != cudaSuccess) break;
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, s->bwd_end[i], s->ar_end[i]) == cudaSuccess) {
      s->exposed_ms += ms > 0.0f ? ms : 0.0f;
      s->exposed_steps++;
    }
    s->read++;
  }
}

}  // namespace pai

using namespace pai;

void pai_dp_destroy(pai_ctx* ctx) {
  if (!ctx->nccl) return;
  if (ctx->nccl->comm) ncclCommDestroy(ctx->nccl->comm);
  if (ctx->nccl->ready) cudaEventDestroy(ctx->nccl->ready);
  if (ctx->nccl->done) cudaEventDestroy(ctx->nccl->done);
  for (int i = 0; i < kStatRing; i++) {
    if (ctx->nccl->bwd_end[i]) cudaEventDestroy(ctx->nccl->bwd_end[i]);
    if (ctx->nccl->ar_end[i]) cudaEventDestroy(ctx->nccl->ar_end[i]);
  }
  delete ctx->nccl;
  ctx->nccl = nullptr;
}

PAI_API pai_status pai_nccl_unique_id(uint8_t id_out[128]) {
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return set_error(PAI_ERR_NCCL, "ncclGetUniqueId failed: %s", ncclGetErrorString(r));
  memcpy(id_out, &id, 128);
  return PAI_OK;
}

PAI_API pai_status pai_nccl_init(pai_ctx* ctx, const uint8_t id[128], int32_t rank, int32_t world, int32_t timeout_ms) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  if (ctx->nccl) return set_error(PAI_ERR_INVALID_OP, "NCCL already initialised on this context");
  if (world < 1 || rank < 0 || rank >= world) return set_error(PAI_ERR_OUT_OF_RANGE, "bad rank %d / world %d", rank, world);
  auto* s = new NcclState();
  s->rank = rank;
  s->world = world;
  s->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  ncclUniqueId uid;
  memcpy(&uid, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = ncclCommInitRankConfig(&s->comm, world, uid, rank, &cfg);
  pai_status st = nccl_wait(s, r, "communicator init");
  if (st != PAI_OK) { delete s; return st; }
  cudaEventCreateWithFlags(&s->ready, cudaEventDisableTiming);
  cudaEventCreateWithFlags(&s->done, cudaEventDisableTiming);
  for (int i = 0; i < kStatRing; i++) {
    cudaEventCreate(&s->bwd_end[i]);
    cudaEventCreate(&s->ar_end[i]);
  }
  ctx->nccl = s;
  return PAI_OK;
}

// Enqueues one group of NCCL calls on the communication stream, ordered after the work queued so far on the compute
// stream; `done` marks its end for pai_allreduce_wait.
template <class Calls>
static pai_status exchange(pai_ctx* ctx, const pai_tensor* tensors, int32_t n, bool shard, const char* what, Calls calls) {
  NcclState* s = ctx->nccl;
  if (!s || !s->comm) return set_error(PAI_ERR_INVALID_OP, "%s without an initialised communicator", what);
  for (int i = 0; i < n; i++) {
    PAI_TRY(check_view(ctx, &tensors[i], "bucket tensor"));
    if (!is_dense(tensors[i])) return set_error(PAI_ERR_ARGUMENT, "%s tensors must be contiguous", what);
    if (shard && numel(tensors[i]) % s->world != 0)
      return set_error(PAI_ERR_ARGUMENT, "%s: %lld elements do not split into %d equal shards", what,
                       (long long)numel(tensors[i]), s->world);
  }
  if (s->world == 1) return PAI_OK;
  PAI_CUDA(cudaEventRecord(s->ready, ctx->stream));
  PAI_CUDA(cudaStreamWaitEvent(ctx->comm_stream, s->ready, 0));
  ncclResult_t r = ncclGroupStart();
  if (r == ncclSuccess) {
    for (int i = 0; i < n && r == ncclSuccess; i++) r = calls(s, tensors[i]);
    ncclResult_t r2 = ncclGroupEnd();
    if (r == ncclSuccess) r = r2;
  }
  PAI_TRY(nccl_wait(s, r, what));
  PAI_CUDA(cudaEventRecord(s->done, ctx->comm_stream));
  s->pending = true;
  return PAI_OK;
}

PAI_API pai_status pai_allreduce_bucket(pai_ctx* ctx, const pai_tensor* tensors, int32_t n) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  return exchange(ctx, tensors, n, false, "all-reduce", [&](NcclState* s, const pai_tensor& t) {
    float* p = fptr(t);
    return ncclAllReduce(p, p, (size_t)numel(t), ncclFloat, ncclSum, s->comm, ctx->comm_stream);
  });
}

// ZeRO-1: rank r owns elements [r·n/W, (r+1)·n/W) of every tensor. The reduce-scatter leaves the cross-rank sum of
// that shard in place (the rest of the tensor is unspecified afterwards); the all-gather copies every rank's shard
// into all ranks' tensors. Both are NCCL's in-place forms (the shard at offset rank x shard size).
PAI_API pai_status pai_reduce_scatter_bucket(pai_ctx* ctx, const pai_tensor* tensors, int32_t n) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  return exchange(ctx, tensors, n, true, "reduce-scatter", [&](NcclState* s, const pai_tensor& t) {
    float* p = fptr(t);
    const size_t shard = (size_t)(numel(t) / s->world);
    return ncclReduceScatter(p, p + shard * (size_t)s->rank, shard, ncclFloat, ncclSum, s->comm, ctx->comm_stream);
  });
}

PAI_API pai_status pai_allgather_bucket(pai_ctx* ctx, const pai_tensor* tensors, int32_t n) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  return exchange(ctx, tensors, n, true, "all-gather", [&](NcclState* s, const pai_tensor& t) {
    float* p = fptr(t);
    const size_t shard = (size_t)(numel(t) / s->world);
    return ncclAllGather(p + shard * (size_t)s->rank, p, shard, ncclFloat, s->comm, ctx->comm_stream);
  });
}

PAI_API pai_status pai_allreduce_wait(pai_ctx* ctx) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  NcclState* s = ctx->nccl;
  if (!s || !s->pending) return PAI_OK;
  s->pending = false;
  read_stats(s);
  if (s->recorded - s->read < kStatRing) {
    const int i = (int)(s->recorded % kStatRing);
    PAI_CUDA(cudaEventRecord(s->bwd_end[i], ctx->stream));
    PAI_CUDA(cudaEventRecord(s->ar_end[i], ctx->comm_stream));
    s->recorded++;
  }
  // The host waits (bounded) for the exchange before the compute stream is ordered after it: a dead peer surfaces
  // here as an error instead of as a compute stream blocked behind a collective that cannot complete.
  PAI_TRY(wait_done(s, s->done));
  PAI_CUDA(cudaStreamWaitEvent(ctx->stream, s->done, 0));
  return PAI_OK;
}

PAI_API pai_status pai_dp_stats(pai_ctx* ctx, double* exposed_ms, int64_t* steps) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  NcclState* s = ctx->nccl;
  double e = 0.0;
  int64_t n = 0;
  if (s) {
    read_stats(s);
    e = s->exposed_ms;
    n = s->exposed_steps;
    s->exposed_ms = 0.0;
    s->exposed_steps = 0;
  }
  if (exposed_ms) *exposed_ms = e;
  if (steps) *steps = n;
  return PAI_OK;
}

PAI_API pai_status pai_nccl_abort(pai_ctx* ctx) {
  if (!ctx) return set_error(PAI_ERR_ARGUMENT, "null context");
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  if (ctx->nccl) abort_comm(ctx->nccl);
  return PAI_OK;
}
