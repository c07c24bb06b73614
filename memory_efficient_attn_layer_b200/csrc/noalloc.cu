// Attention backward for callers that cannot allocate device memory.
//
// mea_attention_backward needs an fp32 dQ accumulator from its caller.  Some
// callers have no way to provide one: a plugin whose execute callback runs
// under a host runtime that forbids (or cannot afford the implicit device
// synchronisation of) cudaMalloc, or code that is handed only its input and
// output buffers and no allocator.  This entry point keeps that accumulator in
// a fixed array compiled into the library instead, and returns dQ in bf16.
//
// Limits and sharing rules:
//  * the array holds MEA_NOALLOC_DQ_MAX_ELEMS fp32 values (16 MiB); every GPU
//    that loads the library holds it until the process exits; problems with
//    B*H*T*N above that are rejected with MEA_ERR_UNSUPPORTED_SHAPE;
//  * every argument is checked before any device work is queued, so a rejected
//    call leaves the stream untouched;
//  * every call uses the same array, which keeps the previous call's
//    contents; each call clears the part it uses before the kernel runs, so
//    calls on one stream are fine, but calls that overlap on the GPU (other
//    streams, other host threads) race on it;
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress); make that first call before any stream capture.
//    The address is cached per device together with the CUDA context it was
//    looked up in; after a cudaDeviceReset the next call looks it up again.
#include <cudaTypedefs.h>

#include <mutex>

#include "launch.h"

#define MEA_NOALLOC_DQ_MAX_ELEMS (4u * 1024u * 1024u)

namespace mea {

static __device__ __align__(256) float g_noalloc_dq[MEA_NOALLOC_DQ_MAX_ELEMS];

// The calling thread's current CUDA context (driver handle), or NULL when the
// driver entry point is unavailable.
static CUcontext current_context() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  });
  CUcontext ctx = nullptr;
  if (fn) fn(&ctx);
  return ctx;
}

// Device address of g_noalloc_dq, looked up once per device (and again after
// the device's context was re-created) with that device current.  In host
// code the array's name is only a stand-in for the symbol.
static int noalloc_scratch(float** out) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  static CUcontext ctx_of[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(MEA_ERR_CUDA, "noalloc: cannot query the current device");
  std::lock_guard<std::mutex> lock(mu);
  const CUcontext ctx = current_context();
  if (!addr[dev] || ctx != ctx_of[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_dq);
    if (e != cudaSuccess || !p)
      return set_error(MEA_ERR_CUDA, "noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
    ctx_of[dev] = current_context();  // the lookup may have created the primary context
  }
  *out = addr[dev];
  return MEA_OK;
}

}  // namespace mea

extern "C" int mea_attention_backward_noalloc(int B, int H, int T, int N, const void* q, const void* k, const void* v,
                                              const void* dO, const float* lse2, const float* delta, void* dq,
                                              void* dk, void* dv, long long ld_dv, int* status, void* stream) {
  using namespace mea;
  if (B <= 0 || H <= 0 || T <= 0 || N <= 0)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "noalloc attention backward: dims must be positive");
  const unsigned long long n = 1ull * B * H * T * N;
  if (n > MEA_NOALLOC_DQ_MAX_ELEMS)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE,
                     "noalloc attention backward: B*H*T*N = %llu exceeds the built-in limit of %u elements "
                     "(use mea_attention_backward with a caller-provided dq accumulator)",
                     n, MEA_NOALLOC_DQ_MAX_ELEMS);
  if (!dq) return set_error(MEA_ERR_INVALID_ARGUMENT, "noalloc attention backward: dq is NULL");
  // dq is written four bf16 values (8 bytes) at a time.
  if (reinterpret_cast<uintptr_t>(dq) & 7)
    return set_error(MEA_ERR_ALIGNMENT, "noalloc attention backward: dq must be 8-byte aligned");
  int rc = check_attn_bwd_args(B, H, T, N, q, k, v, dO, lse2, delta, dk, dv, ld_dv);
  if (rc != MEA_OK) return rc;
  float* acc = nullptr;
  rc = noalloc_scratch(&acc);
  if (rc != MEA_OK) return rc;
  auto st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(acc, 0, n * sizeof(float), st) != cudaSuccess)
    return set_error(MEA_ERR_CUDA, "noalloc attention backward: clearing the accumulator failed");
  rc = run_attn_bwd(B, H, T, N, q, k, v, dO, lse2, delta, acc, dk, dv, ld_dv, status, st);
  if (rc != MEA_OK) return rc;
  return run_cast_f32_bf16(static_cast<long long>(n), acc, dq, st);
}
