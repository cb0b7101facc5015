// ps_b200_block_fwd_static: the single-GPU Wan self-attention block (fused
// q/k RMSNorm + RoPE pre-pass, then attention) for callers that may not
// allocate device memory while they run - for example a plugin host that
// owns the whole device-memory budget through its own pool, or a pipeline
// that must not hit cudaMalloc's implicit device synchronisation mid-step.
//
// Its only scratch - the packed q/k/v buffer between the two kernels and the
// attention kernel's status word - lives in the file-scope array below, of a
// fixed size.  A GPU holds that array from the moment this file's module is
// loaded on it until the process exits: with the default lazy module loading
// that is the first call of this entry point on that GPU; with eager loading
// (CUDA_MODULE_LOADING=EAGER) it is every GPU on which the process creates a
// CUDA context while the library is loaded.  All calls share the array and
// it keeps the last call's contents: the status word is cleared on the
// caller's stream at the start of every call (the packed buffer is fully
// rewritten by the pre-pass), and calls that overlap on the GPU (different
// streams, or other host threads) race on it.
#include "ps_b200.h"
#include "internal.h"

#include <mutex>

namespace psb {
namespace {

constexpr size_t kStatusBytes = 256;
constexpr size_t kQkvBytes = size_t(96) << 20;  // 96 MiB of packed q/k/v

// [0, 256): device status word; [256, 256 + 96 MiB): [3][n][heads][head_dim].
static __device__ __align__(256) unsigned char g_static_scratch[kStatusBytes + kQkvBytes];

std::mutex g_mutex;
struct ScratchSlot {
  CUcontext ctx = nullptr;  // context the address belongs to
  void* ptr = nullptr;
};
ScratchSlot g_scratch[64];

// cuCtxGetCurrent through the runtime's driver entry point (no -lcuda).
CUresult current_context(CUcontext* ctx) {
  using Fn = CUresult (*)(CUcontext*);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(p);
  });
  if (!fn) return CUDA_ERROR_NOT_FOUND;
  return fn(ctx);
}

// Device address of the scratch array on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is queried
// with cudaGetSymbolAddress once per device, with that device current, and
// again whenever the device's context changed since (after cudaDeviceReset,
// or when the primary context was released and created anew, the module is
// loaded again, possibly at another address).
int scratch_address(unsigned char** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_cuda_error("cudaGetDevice", err);
  if (dev < 0 || dev >= 64) return set_error(PS_B200_ERR_UNSUPPORTED, "device index %d above 63", dev);
  // The context current before the lookup (null while the runtime has not
  // made one current on this thread yet).
  CUcontext ctx = nullptr;
  if (current_context(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  ScratchSlot& slot = g_scratch[dev];
  if (!slot.ptr || !ctx || slot.ctx != ctx) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_static_scratch);  // also makes the primary context current
    if (err != cudaSuccess) return set_cuda_error("cudaGetSymbolAddress(static scratch)", err);
    if (current_context(&ctx) != CUDA_SUCCESS || !ctx)
      return set_error(PS_B200_ERR_CUDA, "static block: no current CUDA context on device %d", dev);
    slot.ptr = p;
    slot.ctx = ctx;
  }
  *out = static_cast<unsigned char*>(slot.ptr);
  return PS_B200_OK;
}

}  // namespace
}  // namespace psb

extern "C" int ps_b200_block_fwd_static(const void* x_q, const void* x_k, const void* x_v,
                                        const int64_t x_row_strides[3], const void* w_qnorm,
                                        const void* w_knorm, int w_dtype, const float* freqs,
                                        int64_t freqs_row_stride, void* out, int dtype, int out_dtype, int n,
                                        int heads, int head_dim, float eps, float softmax_scale,
                                        int* host_status, void* stream) {
  using namespace psb;
  if (dtype != PS_B200_BF16 && dtype != PS_B200_FP16)
    return set_error(PS_B200_ERR_UNSUPPORTED, "static block supports bf16 and fp16 inputs only");
  if (n < 0 || heads < 1 || head_dim <= 0) return set_error(PS_B200_ERR_INVALID, "inconsistent block geometry");
  // The attention kernel computes head_dim 128 only: refuse anything else
  // before any work is queued on the shared scratch.
  if (head_dim != 128)
    return set_error(PS_B200_ERR_UNSUPPORTED, "static block supports head_dim 128 only (got %d)", head_dim);
  const size_t need = size_t(3) * size_t(n) * size_t(heads) * size_t(head_dim) * 2;
  if (need > kQkvBytes)
    return set_error(PS_B200_ERR_UNSUPPORTED,
                     "static block needs %zu bytes of scratch for n=%d, heads=%d, head_dim=%d; the static "
                     "scratch holds %zu bytes (n*heads*head_dim <= %zu)",
                     need, n, heads, head_dim, kQkvBytes, kQkvBytes / 6);
  if (host_status) *host_status = 0;
  if (n == 0) return PS_B200_OK;
  unsigned char* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  int* status = reinterpret_cast<int*>(scratch);
  void* qkv = scratch + kStatusBytes;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemsetAsync(status, 0, sizeof(int), s);
  if (err != cudaSuccess) return set_cuda_error("static block: clearing the status word", err);
  if (int rc = ps_b200_prepass(x_q, x_k, x_v, x_row_strides, nullptr, w_qnorm, w_knorm, w_dtype, freqs, freqs_row_stride,
                               qkv, dtype, 1, n, n, heads, heads, head_dim, eps, 1, 0, head_dim / 2, stream))
    return rc;
  if (int rc = ps_b200_ulysses_attn_fwd(qkv, out, dtype, out_dtype, 1, n, n, nullptr, heads, heads, head_dim,
                                        softmax_scale, nullptr, 0, status, stream))
    return rc;
  if (host_status) {
    err = cudaMemcpyAsync(host_status, status, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return set_cuda_error("static block: reading the status word", err);
  }
  return PS_B200_OK;
}
