// HBM-bound kernels around the attention: the fused q/k RMSNorm + RoPE +
// Ulysses pack ("pre-pass") and the receive-side head->sequence unpack.
//
// Pre-pass, one CTA of 256 threads per token row of the send segment and
// batch row (a seg_rows x batch grid):
//   q, k: y = bf16(fp32(x) * rsqrt(mean(x^2) + eps) * w)   (RMSNorm over the
//         full width (Wan, norm_rope 1) or over each head (Flux / H3 QK-norm,
//         norm_rope 2, weight [head_dim] shared by the heads))
//         out[2j], out[2j+1] = F[j] @ (y[2j], y[2j+1])     (interleaved RoPE, style 0)
//         out[j], out[j+P]   = F[j] @ (y[j], y[j+P]), j < P (split-half partial
//         RoPE of H3, style 1; elements >= 2P keep y)
//   v   : copied.
// Each result goes straight to its slot of the all-to-all send buffer
// [world][3][batch][seg_rows][heads_per_rank][head_dim] (the reference's
// [W, T, B, width, h, D] packing): global head g lands in
// destination block g / heads_per_rank at head slot g % heads_per_rank.
// Rows past the local token count and heads past `heads` are written as
// zeros (they are the zero padding of the reference's packing).
// All loads/stores are 16-byte vectors; a token row of q/k stays in registers
// between the sum-of-squares reduction and the normalisation.
#include "ps_b200.h"
#include "internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace psb {
namespace pre {

constexpr int kThreads = 256;

template <bool kFp16>
__device__ __forceinline__ float to_f(uint16_t v) {
  if constexpr (kFp16) {
    return __half2float(__ushort_as_half(v));
  } else {
    return __bfloat162float(__ushort_as_bfloat16(v));
  }
}

template <bool kFp16>
__device__ __forceinline__ uint16_t from_f(float f) {
  if constexpr (kFp16) {
    return __half_as_ushort(__float2half_rn(f));
  } else {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
}

__device__ __forceinline__ void unpack8(const uint4& v, uint16_t (&e)[8]) {
  e[0] = v.x & 0xffff;
  e[1] = v.x >> 16;
  e[2] = v.y & 0xffff;
  e[3] = v.y >> 16;
  e[4] = v.z & 0xffff;
  e[5] = v.z >> 16;
  e[6] = v.w & 0xffff;
  e[7] = v.w >> 16;
}

__device__ __forceinline__ uint4 pack8(const uint16_t (&e)[8]) {
  uint4 v;
  v.x = e[0] | (static_cast<uint32_t>(e[1]) << 16);
  v.y = e[2] | (static_cast<uint32_t>(e[3]) << 16);
  v.z = e[4] | (static_cast<uint32_t>(e[5]) << 16);
  v.w = e[6] | (static_cast<uint32_t>(e[7]) << 16);
  return v;
}

// Sums of two values over the CTA (warp xor-shuffles, then the warp partials
// in warp order).
__device__ __forceinline__ float2 block_sum2(float a, float b, float2* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_float2(a, b);
  __syncthreads();
  float2 s = make_float2(0.f, 0.f);
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    s.x += red[w].x;
    s.y += red[w].y;
  }
  return s;
}

// One CTA per token row.  Every load of the row (q, k and v, kVec 16-byte
// vectors per thread each) is issued before any arithmetic, so the row's
// reads are in flight together; v is stored as soon as it arrives, q and k
// share one block reduction (full-width norm) and one read of the RoPE table.
// At most 64 registers for rows of <= 3 vectors per thread: four CTAs per SM
// keep more rows' loads in flight (9 % faster at configs[1] than three CTAs
// at 80 registers; at 48 registers the spills cost more than the occupancy).
template <bool kFp16, int kVec, bool kSplit>
__global__ void __launch_bounds__(kThreads, kVec >= 4 ? 2 : 4) prepass_kernel(const PrepassArgs a) {
  __shared__ float2 red[kThreads / 32];
  __shared__ uint16_t* sdst[kMaxSegs];
  const int i = blockIdx.x;
  const int b = blockIdx.y;
  const int tid = threadIdx.x;
  if (tid < (a.kv_fanout > a.world ? a.kv_fanout : a.world)) sdst[tid] = static_cast<uint16_t*>(a.dst[tid]);
  __syncthreads();
  const int D = a.head_dim;
  const int h = a.heads_per_rank;
  const int vph = D >> 3;             // vectors per head
  const int nvec = a.heads * vph;     // vectors per token row
  // One kind's [batch][seg_rows][h][D] block; this CTA's row within it.
  const int64_t block_elems = static_cast<int64_t>(a.batch) * a.seg_rows * h * D;
  const int64_t row_off = (static_cast<int64_t>(b) * a.seg_rows + i) * h * D;
  // Destination of vector (head g, element dd) of kind 0; kinds k add k*block_elems.
  auto slot0 = [&](int g, int dd) -> uint16_t* {
    const int dst = g / h;
    const int j = g - dst * h;
    return sdst[dst] + row_off + static_cast<int64_t>(j) * D + dd;
  };
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  // Store one 16-byte vector of `kind` (0 q, 1 k, 2 v) for head g, element dd.
  auto put = [&](int kind, int g, int dd, const uint4& val) {
    if (a.kv_fanout) {
      const int64_t off = row_off + static_cast<int64_t>(g) * D + dd;
      if (kind == 0) {
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.q_out) + off) = val;
      } else {
        for (int d = 0; d < a.kv_fanout; ++d)
          *reinterpret_cast<uint4*>(sdst[d] + (kind - 1) * block_elems + off) = val;
      }
    } else {
      *reinterpret_cast<uint4*>(slot0(g, dd) + kind * block_elems) = val;
    }
  };

  if (i >= a.n_local) {  // token padding of the last ranks: zeros for every head
    const int total = a.world * h * vph;
    for (int kind = 0; kind < 3; ++kind)
      for (int v = tid; v < total; v += kThreads) {
        const int g = v / vph;
        put(kind, g, (v - g * vph) * 8, zero);
      }
    return;
  }

  int gv[kVec], ddv[kVec];
  bool live[kVec];
#pragma unroll
  for (int u = 0; u < kVec; ++u) {
    const int v = tid + u * kThreads;
    live[u] = v < nvec;
    gv[u] = v / vph;
    ddv[u] = (v - gv[u] * vph) * 8;
  }
  uint4 xv[3][kVec];
#pragma unroll
  for (int kind = 0; kind < 3; ++kind) {
    const uint16_t* x = static_cast<const uint16_t*>(a.x[kind]) + static_cast<int64_t>(b) * a.x_batch_stride[kind] +
                        static_cast<int64_t>(i) * a.x_row_stride[kind];
#pragma unroll
    for (int u = 0; u < kVec; ++u)
      if (live[u]) xv[kind][u] = __ldg(reinterpret_cast<const uint4*>(x + gv[u] * a.x_head_stride[kind] + ddv[u]));
  }
#pragma unroll
  for (int u = 0; u < kVec; ++u)
    if (live[u]) put(2, gv[u], ddv[u], xv[2][u]);

  if (a.norm_rope) {
    const bool per_head = a.norm_rope == 2;  // Flux QK-norm: statistic per head, weight [head_dim]
    float ss[2][kVec];
#pragma unroll
    for (int kind = 0; kind < 2; ++kind)
#pragma unroll
      for (int u = 0; u < kVec; ++u) {
        ss[kind][u] = 0.f;
        if (live[u]) {
          uint16_t e[8];
          unpack8(xv[kind][u], e);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float f = to_f<kFp16>(e[q]);
            ss[kind][u] = fmaf(f, f, ss[kind][u]);
          }
        }
      }
    float r[2][kVec];
    if (!per_head) {
      float tq = 0.f, tk = 0.f;
#pragma unroll
      for (int u = 0; u < kVec; ++u) {
        tq += ss[0][u];
        tk += ss[1][u];
      }
      const float2 total = block_sum2(tq, tk, red);
      const float width = static_cast<float>(a.heads * D);
      const float rq = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total.x, width), a.eps)));
      const float rk = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total.y, width), a.eps)));
#pragma unroll
      for (int u = 0; u < kVec; ++u) {
        r[0][u] = rq;
        r[1][u] = rk;
      }
    } else {
      // The vph (= D/8, a power of two <= 32) consecutive lanes holding one
      // head reduce their partial sums with xor shuffles.
#pragma unroll
      for (int kind = 0; kind < 2; ++kind)
#pragma unroll
        for (int u = 0; u < kVec; ++u) {
          float t = ss[kind][u];
          for (int o = vph >> 1; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
          r[kind][u] = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, static_cast<float>(D)), a.eps)));
        }
    }
    const float* frow =
        a.freqs + static_cast<int64_t>(b) * a.freqs_batch_stride + static_cast<int64_t>(i) * a.freqs_row_stride;
    constexpr bool split = kSplit;  // split-half partial RoPE (H3); else interleaved pairs
    const int half_vec = a.rope_pairs >> 3;  // split style: vectors between an element and its partner
    const int lane = tid & 31;
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      const int v = tid + u * kThreads;
      const int dd = ddv[u];
      const int widx = per_head ? dd : v * 8;  // weight element of this vector's first value
      // Split style: the vector holding elements dd..dd+7 pairs with the one
      // rope_pairs elements away, half_vec lanes up or down in the same warp.
      const bool first = split && dd < a.rope_pairs;
      const bool second = split && !first && dd < 2 * a.rope_pairs;
      const int partner_lane = first ? lane + half_vec : (second ? lane - half_vec : lane);
      const int pair0 = split ? (first ? dd : dd - a.rope_pairs) : (dd >> 1);
      const bool rotate = !split || first || second;
      float4 F[4];  // interleaved style: pairs pair0..pair0+3, {F00, F01, F10, F11}, read once for q and k
      if (!split && live[u]) {
        const float4* fp = reinterpret_cast<const float4*>(frow) + pair0;
#pragma unroll
        for (int p = 0; p < 4; ++p) F[p] = __ldg(fp + p);
      }
#pragma unroll
      for (int kind = 0; kind < 2; ++kind) {
        uint16_t e[8];
        unpack8(xv[kind][u], e);
        float y[8];
        if (live[u]) {
          if (a.w_fp32) {
            const float4* wp = reinterpret_cast<const float4*>(static_cast<const float*>(a.w[kind]) + widx);
            const float4 w0 = __ldg(wp), w1 = __ldg(wp + 1);
            const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int q = 0; q < 8; ++q)
              y[q] = to_f<kFp16>(from_f<kFp16>(__fmul_rn(__fmul_rn(to_f<kFp16>(e[q]), r[kind][u]), w[q])));
          } else {
            uint16_t we[8];
            unpack8(__ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.w[kind]) + widx)), we);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              y[q] = to_f<kFp16>(
                  from_f<kFp16>(__fmul_rn(__fmul_rn(to_f<kFp16>(e[q]), r[kind][u]), to_f<kFp16>(we[q]))));
          }
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) y[q] = 0.f;
        }
        uint16_t o[8];
        if (!split) {
          if (live[u]) {
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const float x0 = y[2 * p], x1 = y[2 * p + 1];
              o[2 * p] = from_f<kFp16>(__fadd_rn(__fmul_rn(F[p].x, x0), __fmul_rn(F[p].y, x1)));
              o[2 * p + 1] = from_f<kFp16>(__fadd_rn(__fmul_rn(F[p].z, x0), __fmul_rn(F[p].w, x1)));
            }
          }
        } else {
          // Exchange the normalised (16-bit exact) values with the partner lane;
          // every lane takes part in the shuffles.
          uint16_t yb[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) yb[q] = from_f<kFp16>(y[q]);
          const uint4 mine = pack8(yb);
          uint4 other;
          other.x = __shfl_sync(0xffffffffu, mine.x, partner_lane);
          other.y = __shfl_sync(0xffffffffu, mine.y, partner_lane);
          other.z = __shfl_sync(0xffffffffu, mine.z, partner_lane);
          other.w = __shfl_sync(0xffffffffu, mine.w, partner_lane);
          uint16_t pb[8];
          unpack8(other, pb);
          if (live[u]) {
            if (rotate) {
              const float4* fp = reinterpret_cast<const float4*>(frow) + pair0;
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float4 M = __ldg(fp + q);
                // first half: out_j = M00 x_j + M01 x_{j+P}; second half: out_{j+P} = M10 x_j + M11 x_{j+P}
                const float xj = first ? y[q] : to_f<kFp16>(pb[q]);
                const float xp = first ? to_f<kFp16>(pb[q]) : y[q];
                o[q] = first ? from_f<kFp16>(__fadd_rn(__fmul_rn(M.x, xj), __fmul_rn(M.y, xp)))
                             : from_f<kFp16>(__fadd_rn(__fmul_rn(M.z, xj), __fmul_rn(M.w, xp)));
              }
            } else {
#pragma unroll
              for (int q = 0; q < 8; ++q) o[q] = yb[q];  // past the rotated dims: the normalised value
            }
          }
        }
        if (live[u]) put(kind, gv[u], dd, pack8(o));
      }
    }
  } else {
#pragma unroll
    for (int kind = 0; kind < 2; ++kind)
#pragma unroll
      for (int u = 0; u < kVec; ++u)
        if (live[u]) put(kind, gv[u], ddv[u], xv[kind][u]);
  }
  // Head padding: slots of heads [heads, world*h) are zero.
  const int padded = (a.world * h - a.heads) * vph;
  for (int kind = 0; kind < 3; ++kind)
    for (int v = tid; v < padded; v += kThreads) {
      const int g = a.heads + v / vph;
      put(kind, g, (v % vph) * 8, zero);
    }
}

constexpr int kUnpackThreads = 256;

template <bool kOutFp32, bool kFp16>
__global__ void __launch_bounds__(kUnpackThreads) unpack_kernel(const UnpackArgs a) {
  const int D = a.head_dim;
  const int h = a.heads_per_rank;
  const int vph = D >> 3;
  const int per_token = a.heads * vph;
  const int per_batch = a.n_local * per_token;
  const int total = a.batch * per_batch;
  for (int idx = blockIdx.x * kUnpackThreads + threadIdx.x; idx < total; idx += gridDim.x * kUnpackThreads) {
    const int b = idx / per_batch;
    const int ib = idx - b * per_batch;
    const int i = ib / per_token;
    const int rem = ib - i * per_token;
    const int g = rem / vph;
    const int dd = (rem - g * vph) * 8;
    const int src = g / h;
    const int j = g - src * h;
    const uint16_t* in = static_cast<const uint16_t*>(a.recv) + src * a.src_stride + b * a.batch_stride +
                         i * a.row_stride + static_cast<int64_t>(j) * D + dd;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(in));
    const int64_t o = static_cast<int64_t>(b) * a.out_batch_stride + static_cast<int64_t>(i) * a.out_row_stride +
                      static_cast<int64_t>(g) * D + dd;
    if constexpr (kOutFp32) {
      uint16_t e[8];
      unpack8(v, e);
      float4* out = reinterpret_cast<float4*>(static_cast<float*>(a.out) + o);
      out[0] = make_float4(to_f<kFp16>(e[0]), to_f<kFp16>(e[1]), to_f<kFp16>(e[2]), to_f<kFp16>(e[3]));
      out[1] = make_float4(to_f<kFp16>(e[4]), to_f<kFp16>(e[5]), to_f<kFp16>(e[6]), to_f<kFp16>(e[7]));
    } else {
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + o) = v;
    }
  }
}

// Copies `vectors` 16-byte vectors of src to every destination: each vector
// is read once and stored ndst times (grid-stride, coalesced).
__global__ void __launch_bounds__(256) broadcast_kernel(const BroadcastArgs a) {
  const uint4* src = static_cast<const uint4*>(a.src);
  for (int64_t v = blockIdx.x * 256ll + threadIdx.x; v < a.vectors; v += static_cast<int64_t>(gridDim.x) * 256) {
    const uint4 x = __ldg(src + v);
    for (int d = 0; d < a.ndst; ++d) static_cast<uint4*>(a.dst[d])[v] = x;
  }
}

}  // namespace pre

int launch_prepass(const PrepassArgs& a, bool fp16, cudaStream_t stream) {
  using namespace pre;
  if (a.seg_rows == 0 || a.batch == 0) return 0;
  const dim3 grid(a.seg_rows, a.batch), block(kThreads);
  const int nvec = a.heads * (a.head_dim / 8);
  const int vec = (nvec + kThreads - 1) / kThreads;  // 1..kMaxVec (width <= 8192 is checked by the caller)
  const bool split = a.rope_style == 1 && a.norm_rope != 0;
  switch ((split ? 16 : 0) + (fp16 ? 8 : 0) + vec) {
#define PSB_PREPASS_CASE(code, FP16, VEC, SPLIT) \
  case code: prepass_kernel<FP16, VEC, SPLIT><<<grid, block, 0, stream>>>(a); break;
    PSB_PREPASS_CASE(1, false, 1, false)
    PSB_PREPASS_CASE(2, false, 2, false)
    PSB_PREPASS_CASE(3, false, 3, false)
    PSB_PREPASS_CASE(4, false, 4, false)
    PSB_PREPASS_CASE(9, true, 1, false)
    PSB_PREPASS_CASE(10, true, 2, false)
    PSB_PREPASS_CASE(11, true, 3, false)
    PSB_PREPASS_CASE(12, true, 4, false)
    PSB_PREPASS_CASE(17, false, 1, true)
    PSB_PREPASS_CASE(18, false, 2, true)
    PSB_PREPASS_CASE(19, false, 3, true)
    PSB_PREPASS_CASE(20, false, 4, true)
    PSB_PREPASS_CASE(25, true, 1, true)
    PSB_PREPASS_CASE(26, true, 2, true)
    PSB_PREPASS_CASE(27, true, 3, true)
    PSB_PREPASS_CASE(28, true, 4, true)
#undef PSB_PREPASS_CASE
    default: return set_error(PS_B200_ERR_UNSUPPORTED, "prepass: %d vectors per row", nvec);
  }
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_cuda_error("prepass launch", err);
  count_launch();
  return 0;
}

int launch_broadcast(const BroadcastArgs& a, cudaStream_t stream) {
  using namespace pre;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (a.vectors + 255) / 256;
  const int blocks = static_cast<int>(want < sms * 4LL ? want : sms * 4LL);
  broadcast_kernel<<<blocks, 256, 0, stream>>>(a);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_cuda_error("broadcast launch", err);
  count_launch();
  return 0;
}

int launch_unpack(const UnpackArgs& a, bool fp16, cudaStream_t stream) {
  using namespace pre;
  const int64_t total = static_cast<int64_t>(a.batch) * a.n_local * a.heads * (a.head_dim / 8);
  if (total == 0) return 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (total + kUnpackThreads - 1) / kUnpackThreads;
  const int blocks = static_cast<int>(want < sms * 8LL ? want : sms * 8LL);
  if (a.out_fp32) {
    if (fp16) unpack_kernel<true, true><<<blocks, kUnpackThreads, 0, stream>>>(a);
    else unpack_kernel<true, false><<<blocks, kUnpackThreads, 0, stream>>>(a);
  } else {
    if (fp16) unpack_kernel<false, true><<<blocks, kUnpackThreads, 0, stream>>>(a);
    else unpack_kernel<false, false><<<blocks, kUnpackThreads, 0, stream>>>(a);
  }
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_cuda_error("unpack launch", err);
  count_launch();
  return 0;
}

}  // namespace psb
