// static_scratch.cu — the weight-streaming linear layer for callers that cannot allocate device memory.
//
// Some hosts of this engine cannot call cudaMalloc at all: a simulator or evaluator process that
// runs under a fixed device-memory budget enforced by its own pooling allocator, a plugin loaded
// into such a process, or a real-time control loop that must not allocate after start-up.
// pi05_linear_static gives them the few-token linear layer (out = x . w^T + bias, bf16) without
// any allocation: the split-K partial tiles and the per-tile tickets live in one file-scope
// device array of fixed size, P5_STATIC_SCRATCH_BYTES (16 MiB).  Every GPU that loads this library
// holds that array until the process exits.
//
// Rules for callers:
//   * The first call on each device looks up the array's device address (cudaGetSymbolAddress),
//     raises the kernel's shared-memory limit and fetches the tensor-map encoder.  Make that first
//     call before any stream capture.
//   * All calls share the one array, which keeps the last call's contents.  Calls whose kernels
//     overlap on the GPU (different streams, no ordering between them) race on it.
//   * The tickets are cleared at the start of every call; the partial tiles need no clearing
//     because each is fully written before it is read.
//   * The kernel's waits are bounded.  A wait that gives up records a code in a status word at the
//     front of the array and the output of that call is incomplete; later calls skip their work
//     until pi05_linear_static_status reads the word (after waiting for the stream), clears it and
//     returns PI05_ERR_DEVICE.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "../../include/pi05.h"
#include "gemm_tc.cuh"

using namespace p5;

#define P5_STATIC_SCRATCH_BYTES (16u << 20)
#define P5_STATIC_STATUS_BYTES 256u         // status word of the bounded waits, at the front of the array
#define P5_STATIC_TICKET_BYTES (16u << 10)  // then 4096 tickets, then the partial tiles
#define P5_STATIC_MAX_T 64
#define P5_STATIC_MAX_F 65536
#define P5_STATIC_MAX_K 65536

static __device__ __align__(256) unsigned char g_static_scratch[P5_STATIC_SCRATCH_BYTES];

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceState {
  bool ready = false;
  unsigned char* scratch = nullptr;  // device address of g_static_scratch on this device
  int num_sms = 0;
};

std::mutex g_mu;
DeviceState g_dev[64];
EncodeTiledFn g_encode = nullptr;

int fail(char* err, size_t err_len, int code, const char* msg) {
  if (err && err_len) snprintf(err, err_len, "%s", msg);
  return code;
}

// Once per device, with that device current.
int setup(int dev, char* err, size_t err_len) {
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& s = g_dev[dev];
  if (s.ready) return PI05_OK;
  void* p = nullptr;
  cudaError_t ce = cudaGetSymbolAddress(&p, g_static_scratch);
  if (ce != cudaSuccess || !p) return fail(err, err_len, PI05_ERR_CUDA, "cudaGetSymbolAddress(g_static_scratch) failed");
  ce = cudaFuncSetAttribute(gemm_tc_kernel<64, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            GemmCfg<64>::SMEM);
  if (ce != cudaSuccess) return fail(err, err_len, PI05_ERR_CUDA, "cudaFuncSetAttribute failed");
  if (cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return fail(err, err_len, PI05_ERR_CUDA, "cudaDeviceGetAttribute failed");
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn ||
        q != cudaDriverEntryPointSuccess)
      return fail(err, err_len, PI05_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  s.scratch = static_cast<unsigned char*>(p);
  s.ready = true;
  return PI05_OK;
}

bool tmap(CUtensorMap* m, const void* base, long rows, int K, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" PI05_API int pi05_linear_static(int T, int F, int K, const void* x, const void* w, const void* bias,
                                           void* out, void* stream, char* err, size_t err_len) {
  if (T < 1 || T > P5_STATIC_MAX_T || F < 1 || F > P5_STATIC_MAX_F || K < 8 || K > P5_STATIC_MAX_K || K % 8)
    return fail(err, err_len, PI05_ERR_ARG,
                "pi05_linear_static: needs 1 <= T <= 64, 1 <= F <= 65536, 8 <= K <= 65536, K % 8 == 0");
  if (!x || !w || !out || ((uintptr_t)x & 15) || ((uintptr_t)w & 15) || ((uintptr_t)out & 15) || ((uintptr_t)bias & 1))
    return fail(err, err_len, PI05_ERR_ARG,
                "pi05_linear_static: x, w, out must be 16-byte aligned device pointers, bias 2-byte aligned or NULL");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(err, err_len, PI05_ERR_CUDA, "pi05_linear_static: no current device");
  const int rc = setup(dev, err, err_len);
  if (rc != PI05_OK) return rc;
  const DeviceState& s = g_dev[dev];
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // same tiling as the engine's few-token path: weights on the 128-row MMA side, tokens as N = 64
  GemmArgs ga = {};
  ga.M = F;
  ga.N = T;
  ga.K = K;
  ga.swap = 1;
  ga.tiles_m = (F + 127) / 128;
  ga.tiles_n = 1;
  ga.group_m = 1;
  const int kt = (K + 63) / 64;
  const size_t tile_bytes = (size_t)128 * 64 * 4;
  const int max_partials =
      (int)((P5_STATIC_SCRATCH_BYTES - P5_STATIC_STATUS_BYTES - P5_STATIC_TICKET_BYTES) / tile_bytes);
  int splits = 1;
  if (ga.tiles_m < s.num_sms && kt >= 4) splits = std::max(1, std::min(s.num_sms / ga.tiles_m, kt / 2));
  while (splits > 1 && (splits * ga.tiles_m > max_partials || ga.tiles_m > (int)(P5_STATIC_TICKET_BYTES / 4)))
    --splits;
  const int kper = (kt + splits - 1) / splits;
  ga.splits = (kt + kper - 1) / kper;
  ga.kt_per_split = kper;
  ga.epi = EPI_STORE;
  ga.out = static_cast<bf16*>(out);
  ga.ld_out = F;
  ga.bias = static_cast<const bf16*>(bias);
  ga.out_scale = 1.0f;
  ga.add_mod = 1;
  ga.gate_div = 1;
  ga.status = reinterpret_cast<int*>(s.scratch);
  ga.counters = reinterpret_cast<int*>(s.scratch + P5_STATIC_STATUS_BYTES);
  ga.ws = reinterpret_cast<float*>(s.scratch + P5_STATIC_STATUS_BYTES + P5_STATIC_TICKET_BYTES);
  ga.pdl = 0;

  CUtensorMap ta, tb;
  if (!tmap(&ta, w, F, K, 128) || !tmap(&tb, x, T, K, 64))
    return fail(err, err_len, PI05_ERR_ARG, "pi05_linear_static: tensor map rejected the operands");
  if (cudaMemsetAsync(s.scratch + P5_STATIC_STATUS_BYTES, 0, P5_STATIC_TICKET_BYTES, st) != cudaSuccess)
    return fail(err, err_len, PI05_ERR_CUDA, "pi05_linear_static: clearing the tickets failed");
  const int units = ga.tiles_m * ga.splits;
  gemm_tc_kernel<64, EPI_STORE><<<dim3(std::min(units, s.num_sms)), 256, GemmCfg<64>::SMEM, st>>>(ta, tb, ga);
  const cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) return fail(err, err_len, PI05_ERR_CUDA, cudaGetErrorString(ce));
  return PI05_OK;
}

// Waits for `stream`, then reads and clears the status word that the kernel's bounded waits write.
extern "C" PI05_API int pi05_linear_static_status(void* stream, char* err, size_t err_len) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(err, err_len, PI05_ERR_CUDA, "pi05_linear_static_status: no current device");
  const int rc = setup(dev, err, err_len);
  if (rc != PI05_OK) return rc;
  const DeviceState& s = g_dev[dev];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t ce = cudaStreamSynchronize(st);
  if (ce != cudaSuccess) return fail(err, err_len, PI05_ERR_CUDA, cudaGetErrorString(ce));
  int word = 0;
  ce = cudaMemcpy(&word, s.scratch, sizeof(int), cudaMemcpyDeviceToHost);
  if (ce != cudaSuccess) return fail(err, err_len, PI05_ERR_CUDA, cudaGetErrorString(ce));
  if (word == 0) return PI05_OK;
  if (cudaMemset(s.scratch, 0, sizeof(int)) != cudaSuccess)
    return fail(err, err_len, PI05_ERR_CUDA, "pi05_linear_static_status: clearing the status word failed");
  char msg[128];
  snprintf(msg, sizeof msg, "pi05_linear_static: a device-side wait gave up (status %d); that call's output is incomplete",
           word);
  return fail(err, err_len, PI05_ERR_DEVICE, msg);
}
