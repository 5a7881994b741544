// Data parallelism: one process per GPU, gradient buckets summed with NCCL all-reduce on a dedicated stream so the
// exchange of one transformer block's gradients overlaps the backward of the blocks before it.
// The reference is single-device; this is the data-parallel extension of its trainer.
// The communicator is created non-blocking and every NCCL call is polled under a host deadline, so a dead peer
// ends in PAI_ERR_NCCL / PAI_ERR_TIMEOUT (after ncclCommAbort) instead of a hang.
#include <nccl.h>

#include <chrono>
#include <thread>

#include "common.cuh"

namespace pai {

struct NcclState {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  int timeout_ms = 60000;
  cudaEvent_t ready = nullptr;  // compute stream -> comm stream
  cudaEvent_t done = nullptr;   // comm stream -> compute stream
  bool pending = false;
};

static pai_status nccl_wait(NcclState* s, ncclResult_t r, const char* what) {
  auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(s->timeout_ms);
  while (r == ncclInProgress) {
    if (std::chrono::steady_clock::now() > deadline) {
      ncclCommAbort(s->comm);
      s->comm = nullptr;
      return set_error(PAI_ERR_TIMEOUT, "NCCL %s did not complete within %d ms; communicator aborted", what, s->timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    ncclCommGetAsyncError(s->comm, &r);
  }
  if (r != ncclSuccess) {
    if (s->comm) { ncclCommAbort(s->comm); s->comm = nullptr; }
    return set_error(PAI_ERR_NCCL, "NCCL %s failed: %s", what, ncclGetErrorString(r));
  }
  return PAI_OK;
}

}  // namespace pai

using namespace pai;

void pai_dp_destroy(pai_ctx* ctx) {
  if (!ctx->nccl) return;
  if (ctx->nccl->comm) ncclCommDestroy(ctx->nccl->comm);
  if (ctx->nccl->ready) cudaEventDestroy(ctx->nccl->ready);
  if (ctx->nccl->done) cudaEventDestroy(ctx->nccl->done);
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
  ctx->nccl = s;
  return PAI_OK;
}

PAI_API pai_status pai_allreduce_bucket(pai_ctx* ctx, const pai_tensor* tensors, int32_t n) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  NcclState* s = ctx->nccl;
  if (!s || !s->comm) return set_error(PAI_ERR_INVALID_OP, "all-reduce without an initialised communicator");
  for (int i = 0; i < n; i++) {
    PAI_TRY(check_view(ctx, &tensors[i], "bucket tensor"));
    if (!is_dense(tensors[i])) return set_error(PAI_ERR_ARGUMENT, "all-reduce tensors must be contiguous");
  }
  if (s->world == 1) return PAI_OK;
  PAI_CUDA(cudaEventRecord(s->ready, ctx->stream));
  PAI_CUDA(cudaStreamWaitEvent(ctx->comm_stream, s->ready, 0));
  ncclResult_t r = ncclGroupStart();
  if (r == ncclSuccess) {
    for (int i = 0; i < n && r == ncclSuccess; i++) {
      float* p = fptr(tensors[i]);
      r = ncclAllReduce(p, p, (size_t)numel(tensors[i]), ncclFloat, ncclSum, s->comm, ctx->comm_stream);
    }
    ncclResult_t r2 = ncclGroupEnd();
    if (r == ncclSuccess) r = r2;
  }
  PAI_TRY(nccl_wait(s, r, "all-reduce"));
  PAI_CUDA(cudaEventRecord(s->done, ctx->comm_stream));
  s->pending = true;
  return PAI_OK;
}

PAI_API pai_status pai_allreduce_wait(pai_ctx* ctx) {
  PAI_TRY(enter(ctx));
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  NcclState* s = ctx->nccl;
  if (!s || !s->pending) return PAI_OK;
  PAI_CUDA(cudaStreamWaitEvent(ctx->stream, s->done, 0));
  s->pending = false;
  return PAI_OK;
}

PAI_API pai_status pai_nccl_abort(pai_ctx* ctx) {
  if (!ctx) return set_error(PAI_ERR_ARGUMENT, "null context");
  std::lock_guard<std::recursive_mutex> lk(ctx->mu);
  if (ctx->nccl && ctx->nccl->comm) {
    ncclCommAbort(ctx->nccl->comm);
    ctx->nccl->comm = nullptr;
  }
  return PAI_OK;
}
