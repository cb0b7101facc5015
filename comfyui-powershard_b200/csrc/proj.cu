// Projection GEMMs of the Wan self-attention block on sm_100a (tcgen05 +
// TMEM + TMA), with the step that follows or precedes each one fused in.
//
//   epi 1 (q/k/v projection): [q|k|v] = x [Wq|Wk|Wv]^T + b.  The epilogue of
//     a q or k tile applies RMSNorm over the full projection width, the norm
//     weight and the interleaved RoPE, and every tile stores its rows
//     straight into the Ulysses send layout [dst][3][seg_rows][h][D] (or the
//     peers' receive buffers), so the projections never reach HBM.
//   epi 0 (output projection): y = A Wo^T + b, with A read in place from the
//     exchange buffer that holds the attention output - the peer exchange's
//     staging rows, or the NCCL receive buffer's per-source blocks (a_mode 1)
//     - so no unpack pass runs before the GEMM.
//
// The row statistic of RMSNorm spans all width/256 column tiles of a row
// block, which run on different CTAs.  The kernel is persistent (one CTA per
// SM, cooperative launch: every CTA resident) and works in rounds; a round
// holds whole q/k groups (the width/256 tiles of one row block's q or k),
// so all tiles of a group are in flight at once.  Each posts its per-row
// partial sum of squares and bumps the group's counter; once the counter
// reaches the group size, every tile adds the partials in a fixed order (the
// same bits on every tile and every run) and normalises.  v tiles and, with
// epi 0, all tiles have no such dependence and fill the remaining slots.
//
// Warp roles (192 threads): warps 0-3 epilogue (thread = one row of the
// tile, TMEM lane), warp 4 TMA producer (4-stage ring of 128x64 A and
// 256x64 B tiles, 128-byte swizzle), warp 5 TMEM allocation + UMMA issuer
// (M=128 N=256 K=16, fp32 accumulators, two 256-column TMEM buffers so the
// epilogue of one tile overlaps the main loop of the next).  Every wait,
// including the wait for a group's partials, is bounded.
#include "ptx.cuh"
#include "ps_b200.h"
#include "internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace psb {
namespace proj {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kAStage = kBM * kBK * 2;  // 16 KiB
constexpr int kBStage = kBN * kBK * 2;  // 32 KiB
constexpr int kThreads = 192;
constexpr int kSmemBarOff = kStages * (kAStage + kBStage);
enum Bar : int {
  kFull = 0,
  kEmpty = kFull + kStages,
  kAccFull = kEmpty + kStages,
  kAccEmpty = kAccFull + 2,
  kDrain = kAccEmpty + 2,
  kNumBars = kDrain + 1
};
constexpr int kSmemBytes = kSmemBarOff + 256 + 1024;
static_assert(kNumBars * 8 + 8 <= 256, "barrier block overflow");

enum Err : int {
  kErrFull = 131,
  kErrEmpty = 132,
  kErrAcc = 133,
  kErrGroup = 134,
  kErrDrain = 135,
};

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

// One task: a 128 x 256 output tile of one projection.
struct Task {
  bool valid;
  int kind;   // 0 q, 1 k, 2 v (epi 1); 0 (epi 0)
  int rb;     // row block
  int tile;   // column tile within the projection
  int group;  // epi 1, q/k: rb * 2 + kind
};

// Task of CTA c in round r (P CTAs).  epi 1: round r < rg holds whole q/k
// groups in its first ng * G slots and v tiles after them; later rounds
// hold only v tiles.  epi 0: tiles in order.
__device__ __forceinline__ Task task_of(const ProjArgs& a, int r, int c, int P) {
  Task t{false, 0, 0, 0, 0};
  const int G = a.ntile_n;
  if (a.epi == 0) {
    const int idx = r * P + c;
    if (idx < a.total_tiles) {
      t.valid = true;
      t.rb = idx / G;
      t.tile = idx - t.rb * G;
    }
    return t;
  }
  const int gpr = a.groups_per_round;
  const int rg = (a.total_groups + gpr - 1) / gpr;
  int vidx;
  if (r < rg) {
    const int g0 = r * gpr;
    const int ng = min(gpr, a.total_groups - g0);
    if (c < ng * G) {
      t.valid = true;
      t.group = g0 + c / G;
      t.tile = c - (c / G) * G;
      t.kind = t.group & 1;
      t.rb = t.group >> 1;
      return t;
    }
    vidx = r * P - g0 * G + (c - ng * G);
  } else {
    vidx = rg * P - a.total_groups * G + (r - rg) * P + c;
  }
  if (vidx < a.total_tiles) {
    t.valid = true;
    t.kind = 2;
    t.rb = vidx / G;
    t.tile = vidx - t.rb * G;
  }
  return t;
}

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int code) {
  bool ok = mbar_wait(bar, parity, abort_flag, status, code);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, int* status) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      if (status) atomicCAS(status, 0, kErrDrain);
      return;
    }
  }
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 32 consecutive bias / weight values of column col (fp32 or 16-bit), 0 if absent.
template <bool kFp16>
__device__ __forceinline__ void load32(const void* p, int fp32, int col, float (&v)[32]) {
  if (!p) {
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = 0.f;
    return;
  }
  if (fp32) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + col);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float4 f = __ldg(q + u);
      v[4 * u] = f.x;
      v[4 * u + 1] = f.y;
      v[4 * u + 2] = f.z;
      v[4 * u + 3] = f.w;
    }
  } else {
    const uint4* q = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + col);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint4 w = __ldg(q + u);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        v[8 * u + 2 * h] = to_f<kFp16>(static_cast<uint16_t>(ws[h] & 0xffffu));
        v[8 * u + 2 * h + 1] = to_f<kFp16>(static_cast<uint16_t>(ws[h] >> 16));
      }
    }
  }
}

template <bool kFp16>
__device__ __forceinline__ void store32_16(uint16_t* dst, const float (&y)[32]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint4 w;
    w.x = from_f<kFp16>(y[8 * u + 0]) | (static_cast<uint32_t>(from_f<kFp16>(y[8 * u + 1])) << 16);
    w.y = from_f<kFp16>(y[8 * u + 2]) | (static_cast<uint32_t>(from_f<kFp16>(y[8 * u + 3])) << 16);
    w.z = from_f<kFp16>(y[8 * u + 4]) | (static_cast<uint32_t>(from_f<kFp16>(y[8 * u + 5])) << 16);
    w.w = from_f<kFp16>(y[8 * u + 6]) | (static_cast<uint32_t>(from_f<kFp16>(y[8 * u + 7])) << 16);
    reinterpret_cast<uint4*>(dst)[u] = w;
  }
}

template <bool kFp16>
__global__ void __launch_bounds__(kThreads, 1)
    proj_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w0,
                const __grid_constant__ CUtensorMap tm_w1, const __grid_constant__ CUtensorMap tm_w2,
                const ProjArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kAStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int P = gridDim.x;
  const int c = blockIdx.x;
  const int ksteps = a.kdim / kBK;
  int* status = a.status;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kFull + s), 1);
      mbar_init(bar(kEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kAccFull + b), 1);
      mbar_init(bar(kAccEmpty + b), 4);
    }
    mbar_init(bar(kDrain), 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_w0);
      int it = 0;
      bool ok = true;
      for (int r = 0; r < a.rounds && ok; ++r) {
        const Task t = task_of(a, r, c, P);
        if (!t.valid) continue;
        const CUtensorMap* mw = t.kind == 0 ? &tm_w0 : (t.kind == 1 ? &tm_w1 : &tm_w2);
        const int row0 = t.rb * kBM, n0 = t.tile * kBN;
        for (int kk = 0; kk < ksteps; ++kk, ++it) {
          const int s = it % kStages;
          if (it >= kStages) {
            ok = mbar_wait(bar(kEmpty + s), ((it / kStages) - 1) & 1u, abort_flag, status, kErrEmpty);
            if (!ok) break;
          }
          mbar_arrive_expect_tx(bar(kFull + s), kAStage + kBStage);
          const int k0 = kk * kBK;
          if (a.a_mode == 0) {
            tma_load_2d(smem_u32(sA + s * kAStage), &tm_a, bar(kFull + s), k0, row0);
          } else {
            const int src = k0 / a.a_block_k;
            tma_load_3d(smem_u32(sA + s * kAStage), &tm_a, bar(kFull + s), k0 - src * a.a_block_k, row0, src);
          }
          tma_load_2d(smem_u32(sB + s * kBStage), mw, bar(kFull + s), k0, n0);
        }
      }
      // Every copy issued lands before the CTA may exit.
      for (int j = max(0, it - kStages); j < it; ++j) drain_wait(bar(kFull + j % kStages), (j / kStages) & 1u, status);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, kBN, !kFp16, false, false);
      const uint64_t da = sdesc_sw128(smem_u32(sA), 16, 1024);
      const uint64_t db = sdesc_sw128(smem_u32(sB), 16, 1024);
      int it = 0, seq = 0;
      bool ok = true;
      for (int r = 0; r < a.rounds && ok; ++r) {
        const Task t = task_of(a, r, c, P);
        if (!t.valid) continue;
        const int b = seq & 1;
        if (seq >= 2) {
          ok = mbar_wait(bar(kAccEmpty + b), ((seq >> 1) - 1) & 1u, abort_flag, status, kErrAcc);
          if (!ok) break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + b * kBN;
        for (int kk = 0; kk < ksteps; ++kk, ++it) {
          const int s = it % kStages;
          ok = mbar_wait(bar(kFull + s), (it / kStages) & 1u, abort_flag, status, kErrFull);
          if (!ok) break;
          tc_fence_after();
          const uint64_t das = da + static_cast<uint64_t>((s * kAStage) >> 4);
          const uint64_t dbs = db + static_cast<uint64_t>((s * kBStage) >> 4);
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j)
            umma_ss(acc, das + ((32 * j) >> 4), dbs + ((32 * j) >> 4), idesc, (kk | j) != 0 ? 1u : 0u);
          umma_commit(bar(kEmpty + s));
        }
        if (!ok) break;
        umma_commit(bar(kAccFull + b));
        ++seq;
      }
      umma_commit(bar(kDrain));
      drain_wait(bar(kDrain), 0, status);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 0-3)
    const int row = warp * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const int G = a.ntile_n;
    const int D = a.head_dim, h = a.heads_per_rank;
    int seq = 0;
    bool ok = true;
    for (int r = 0; r < a.rounds; ++r) {
      const Task t = task_of(a, r, c, P);
      if (!t.valid) continue;
      const int b = seq & 1;
      ++seq;
      if (ok) ok = warp_wait(bar(kAccFull + b), ((seq - 1) >> 1) & 1u, abort_flag, status, kErrAcc);
      tc_fence_after();
      const uint32_t acc = tmem + lane_off + b * kBN;
      const int m = t.rb * kBM + row;  // GEMM row
      const bool live = m < a.n;
      // epi 1: batch row and token of GEMM row m; epi 0: the token itself.
      const int bi = a.epi == 1 ? m / a.n_local : 0;
      const int token = a.epi == 1 ? m - bi * a.n_local : m;
      const int n0 = t.tile * kBN;
      const void* bias = a.bias[t.kind];
      if (a.epi == 0) {
        // y = A W^T + b, stored row-major (fp32 or the 16-bit type).
        if (ok) {
#pragma unroll 1
          for (int ch = 0; ch < kBN / 32; ++ch) {
            uint32_t v[32];
            tmem_ld32(acc + ch * 32, v);
            tmem_wait_ld();
            float bv[32];
            load32<kFp16>(bias, a.bias_fp32, n0 + ch * 32, bv);
            float y[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) y[e] = __uint_as_float(v[e]) + bv[e];
            if (live) {
              const int64_t off = static_cast<int64_t>(token) * a.out_row_stride + n0 + ch * 32;
              if (a.out_fp32) {
                float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
#pragma unroll
                for (int u = 0; u < 8; ++u) dst[u] = make_float4(y[4 * u], y[4 * u + 1], y[4 * u + 2], y[4 * u + 3]);
              } else {
                store32_16<kFp16>(static_cast<uint16_t*>(a.out) + off, y);
              }
            }
          }
        }
      } else {
        float rnorm = 1.f;
        if (t.kind < 2) {
          // Pass 1: this tile's part of the row's sum of squares.
          float ss = 0.f;
          if (ok) {
#pragma unroll 1
            for (int ch = 0; ch < kBN / 32; ++ch) {
              uint32_t v[32];
              tmem_ld32(acc + ch * 32, v);
              tmem_wait_ld();
              float bv[32];
              load32<kFp16>(bias, a.bias_fp32, n0 + ch * 32, bv);
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                const float x = __uint_as_float(v[e]) + bv[e];
                ss = fmaf(x, x, ss);
              }
            }
          }
          float* part = a.ss_part + static_cast<int64_t>(t.group) * G * kBM;
          part[t.tile * kBM + row] = ss;
          __threadfence();  // every writer's partial is visible GPU-wide before the group counter moves
          named_bar_sync(1, 128);
          // One thread posts this tile and waits until all G tiles of the
          // group have posted (bounded), then every thread sums the G
          // partials of its row in tile order.
          if (threadIdx.x == 0) {
            __threadfence();
            red_release_gpu_add(a.counters + t.group, 1u);
            const uint64_t t0 = globaltimer();
            bool waited = true;
            while (ld_acquire_gpu(a.counters + t.group) < static_cast<unsigned>(G)) {
              if (*abort_flag || globaltimer() - t0 > kWaitLimitNs) {
                waited = false;
                break;
              }
            }
            if (!waited) {
              *abort_flag = 1;
              if (status) atomicCAS(status, 0, kErrGroup);
            }
          }
          named_bar_sync(1, 128);
          float sum = 0.f;
          for (int j = 0; j < G; ++j) sum += __ldcg(part + j * kBM + row);
          rnorm = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(a.width)), a.eps)));
        }
        // Pass 2: (q/k) normalise, weight, rotate; store to the send layout.
        if (ok) {
          const void* nw = t.kind < 2 ? a.normw[t.kind] : nullptr;
          const float* frow = a.freqs + (live ? bi * a.freqs_batch_stride + static_cast<int64_t>(token) *
                                                                                  a.freqs_row_stride : 0);
#pragma unroll 1
          for (int ch = 0; ch < kBN / 32; ++ch) {
            uint32_t v[32];
            tmem_ld32(acc + ch * 32, v);
            tmem_wait_ld();
            float bv[32];
            load32<kFp16>(bias, a.bias_fp32, n0 + ch * 32, bv);
            const int col = n0 + ch * 32;
            const int g = col / D;
            const int d0 = col - g * D;
            float y[32];
            if (t.kind < 2) {
              float w[32];
              load32<kFp16>(nw, a.normw_fp32, col, w);
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                const float x = __uint_as_float(v[e]) + bv[e];
                y[e] = to_f<kFp16>(from_f<kFp16>(__fmul_rn(__fmul_rn(x, rnorm), w[e])));
              }
              if (live) {
                const float4* fp = reinterpret_cast<const float4*>(frow) + (d0 >> 1);
#pragma unroll
                for (int p = 0; p < 16; ++p) {
                  const float4 F = __ldg(fp + p);
                  const float x0 = y[2 * p], x1 = y[2 * p + 1];
                  y[2 * p] = __fadd_rn(__fmul_rn(F.x, x0), __fmul_rn(F.y, x1));
                  y[2 * p + 1] = __fadd_rn(__fmul_rn(F.z, x0), __fmul_rn(F.w, x1));
                }
              }
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) y[e] = __uint_as_float(v[e]) + bv[e];
            }
            if (live) {
              const int dest = g / h;
              const int slot = g - dest * h;
              uint16_t* dst = static_cast<uint16_t*>(a.dst[dest]) +
                              (((static_cast<int64_t>(t.kind) * a.batch + bi) * a.seg_rows + token) * h + slot) * D + d0;
              store32_16<kFp16>(dst, y);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kAccEmpty + b));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Zero padding of the send layout: token rows [n_local, seg_rows) of every
// slot and head slots [heads, world * h) of rows [0, n_local), for the three
// kinds and every batch row.
__global__ void __launch_bounds__(256) pad_kernel(const ProjArgs a) {
  const int D = a.head_dim, h = a.heads_per_rank;
  const int vph = D / 8;
  const int64_t slots_per_row = static_cast<int64_t>(a.world) * h;
  const int64_t pad_rows = static_cast<int64_t>(a.seg_rows - a.n_local) * slots_per_row;  // padding rows, all slots
  const int64_t pad_heads = static_cast<int64_t>(a.n_local) * (slots_per_row - a.heads);  // padded slots of live rows
  const int64_t per_kb = (pad_rows + pad_heads) * vph;  // one (kind, batch row)
  const int64_t total = 3 * static_cast<int64_t>(a.batch) * per_kb;
  for (int64_t v = blockIdx.x * 256ll + threadIdx.x; v < total; v += static_cast<int64_t>(gridDim.x) * 256) {
    const int64_t kb = v / per_kb;  // kind * batch + b
    int64_t u = v - kb * per_kb;
    const int dd = static_cast<int>(u % vph) * 8;
    u /= vph;
    int token, g;
    if (u < pad_rows) {
      token = a.n_local + static_cast<int>(u / slots_per_row);
      g = static_cast<int>(u % slots_per_row);
    } else {
      u -= pad_rows;
      const int per = static_cast<int>(slots_per_row - a.heads);
      token = static_cast<int>(u / per);
      g = a.heads + static_cast<int>(u % per);
    }
    const int dest = g / h;
    const int slot = g - dest * h;
    uint16_t* dst = static_cast<uint16_t*>(a.dst[dest]) + ((kb * a.seg_rows + token) * h + slot) * D + dd;
    *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
  }
}

}  // namespace proj

namespace {
template <bool kFp16>
int prepare_proj() {
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (done[dev]) return 0;
  const cudaError_t err = cudaFuncSetAttribute(proj::proj_kernel<kFp16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               proj::kSmemBytes);
  if (err != cudaSuccess) return set_cuda_error("projection: cudaFuncSetAttribute", err);
  done[dev] = true;
  return 0;
}
}  // namespace

int launch_proj(const CUtensorMap& ta, const CUtensorMap& tw0, const CUtensorMap& tw1, const CUtensorMap& tw2,
                const ProjArgs& args, bool fp16, int ctas, cudaStream_t stream) {
  using namespace proj;
  if (args.epi == 1) {
    const int64_t pads = (static_cast<int64_t>(args.seg_rows - args.n_local) * args.world * args.heads_per_rank +
                          static_cast<int64_t>(args.n_local) * (args.world * args.heads_per_rank - args.heads));
    if (pads > 0) {
      const int64_t vecs = 3 * int64_t(args.batch) * pads * (args.head_dim / 8);
      const int blocks = static_cast<int>(vecs / 256 + 1 < 4096 ? vecs / 256 + 1 : 4096);
      pad_kernel<<<blocks, 256, 0, stream>>>(args);
      cudaError_t err = cudaGetLastError();
      if (err != cudaSuccess) return set_cuda_error("projection padding launch", err);
      count_launch();
    }
  }
  if (args.rounds <= 0) return 0;
  void* params[] = {const_cast<CUtensorMap*>(&ta), const_cast<CUtensorMap*>(&tw0), const_cast<CUtensorMap*>(&tw1),
                    const_cast<CUtensorMap*>(&tw2), const_cast<ProjArgs*>(&args)};
  cudaError_t err;
  if (fp16) {
    if (int rc = prepare_proj<true>()) return rc;
    err = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(proj_kernel<true>), dim3(ctas), dim3(kThreads),
                                      params, kSmemBytes, stream);
  } else {
    if (int rc = prepare_proj<false>()) return rc;
    err = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(proj_kernel<false>), dim3(ctas), dim3(kThreads),
                                      params, kSmemBytes, stream);
  }
  if (err != cudaSuccess) return set_cuda_error("projection launch", err);
  count_launch();
  return 0;
}

}  // namespace psb
