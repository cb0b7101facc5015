// ps_b200_block_fwd_static: the single-GPU Wan self-attention block (fused
// q/k RMSNorm + RoPE pre-pass, then attention) for callers that may not
// allocate device memory while they run - for example a plugin host that
// owns the whole device-memory budget through its own pool, or a pipeline
// that must not hit cudaMalloc's implicit device synchronisation mid-step.
//
// Its only scratch - the packed q/k/v buffer between the two kernels and the
// attention kernel's status word - lives in the file-scope array below, of a
// fixed size.  Every GPU on which this entry point is used holds that array
// until the process exits.  All calls share it and it keeps the last call's
// contents: the status word is cleared on the caller's stream at the start of
// every call (the packed buffer is fully rewritten by the pre-pass), and calls
// that overlap on the GPU (different streams, or other host threads) race on
// it.
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
void* g_scratch_ptr[64] = {nullptr};

// Device address of the scratch array on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is queried
// with cudaGetSymbolAddress once per device (with that device current).
int scratch_address(unsigned char** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_cuda_error("cudaGetDevice", err);
  if (dev < 0 || dev >= 64) return set_error(PS_B200_ERR_UNSUPPORTED, "device index %d above 63", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_static_scratch);
    if (err != cudaSuccess) return set_cuda_error("cudaGetSymbolAddress(static scratch)", err);
    g_scratch_ptr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_ptr[dev]);
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
