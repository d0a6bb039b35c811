// dp_nccl.cuh — data-parallel LoRA over NCCL: the one exchange step of the train step (the adapter
// gradients of every rank averaged before the identical clip + AdamW on each rank).  The reference
// trained on one GPU (docs/archive/windows/π05_네이티브엔진.md:464); the exchange follows the LoRA step's
// data-parallel plan: one flat fp32 gradient buffer, averaged per layer as soon as the backward pass has
// finished that layer, on a communication stream ordered by CUDA events, with no host synchronisation.
//
// NCCL is resolved at run time from the process (dlopen of libnccl.so.2: the copy a host framework such
// as torch already loaded, else the system one), so the library loads and runs single-GPU without it.
// Communicators are created non-blocking and every wait on them is bounded (PI05_NCCL_TIMEOUT_S,
// default 120 s): a rank that never joins ends the attach with an error instead of a hang.
#pragma once
#include <dlfcn.h>
#include <nccl.h>  // types and constants only; the functions are looked up in the loaded library

#include <chrono>
#include <thread>

namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi& nccl_api() {
  static NcclApi api;
  static bool tried = false;
  if (tried) return api;
  tried = true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);  // a copy already in the process
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    api.why = std::string("libnccl.so.2 not found: ") + dlerror();
    return api;
  }
  auto sym = [&](const char* n) { return dlsym(h, n); };
  api.get_unique_id = (decltype(api.get_unique_id))sym("ncclGetUniqueId");
  api.init_rank_config = (decltype(api.init_rank_config))sym("ncclCommInitRankConfig");
  api.all_reduce = (decltype(api.all_reduce))sym("ncclAllReduce");
  api.comm_destroy = (decltype(api.comm_destroy))sym("ncclCommDestroy");
  api.comm_abort = (decltype(api.comm_abort))sym("ncclCommAbort");
  api.async_error = (decltype(api.async_error))sym("ncclCommGetAsyncError");
  api.error_string = (decltype(api.error_string))sym("ncclGetErrorString");
  api.ok = api.get_unique_id && api.init_rank_config && api.all_reduce && api.comm_destroy && api.comm_abort &&
           api.async_error && api.error_string;
  if (!api.ok) api.why = "libnccl.so.2 lacks a needed entry point";
  return api;
}

double nccl_timeout_s() {
  const char* s = getenv("PI05_NCCL_TIMEOUT_S");
  const double v = s ? atof(s) : 120.0;
  return v > 0 ? v : 120.0;
}

// Waits (bounded) until a non-blocking communicator has finished its pending operation.
bool nccl_settle(pi05_engine* e, ncclComm_t comm, const char* what) {
  NcclApi& A = nccl_api();
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    if (A.async_error(comm, &st) != ncclSuccess) return set_err(e, std::string(what) + ": ncclCommGetAsyncError failed");
    if (st == ncclSuccess) return true;
    if (st != ncclInProgress) return set_err(e, std::string(what) + ": " + A.error_string(st));
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > nccl_timeout_s())
      return set_err(e, std::string(what) + ": timed out (a rank did not join)");
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

// The communicator of a data-parallel LoRA engine and its stream and events.
struct DpComm {
  ncclComm_t comm = nullptr;
  cudaStream_t cs = nullptr;
  int rank = 0, world = 1;
  std::vector<cudaEvent_t> layer_done;  // per layer: its gradients are final on the engine stream
  cudaEvent_t reduced = nullptr;        // the exchange of the step is enqueued on cs
};

void dp_release(DpComm* d) {
  if (!d) return;
  if (d->cs) cudaStreamSynchronize(d->cs);
  if (d->comm) nccl_api().comm_destroy(d->comm);
  for (cudaEvent_t ev : d->layer_done) cudaEventDestroy(ev);
  if (d->reduced) cudaEventDestroy(d->reduced);
  if (d->cs) cudaStreamDestroy(d->cs);
  delete d;
}

// Average `count` floats at `p` over the ranks, on the communication stream after event `after` (or
// after everything queued on the engine stream when null).
bool dp_average(pi05_engine* e, DpComm* d, float* p, size_t count, cudaEvent_t after) {
  NcclApi& A = nccl_api();
  if (!after) {
    CK(cudaEventRecord(d->reduced, e->stream));
    after = d->reduced;
  }
  CK(cudaStreamWaitEvent(d->cs, after, 0));
  const ncclResult_t r = A.all_reduce(p, p, count, ncclFloat32, ncclAvg, d->comm, d->cs);
  if (r != ncclSuccess && r != ncclInProgress) return set_err(e, std::string("ncclAllReduce: ") + A.error_string(r));
  return nccl_settle(e, d->comm, "ncclAllReduce");
}

// The engine stream waits for the exchanges enqueued so far.
bool dp_join(pi05_engine* e, DpComm* d) {
  CK(cudaEventRecord(d->reduced, d->cs));
  CK(cudaStreamWaitEvent(e->stream, d->reduced, 0));
  return true;
}

}  // namespace
