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
// Two-SM tiles: a cluster of two CTAs computes one 256 x 256 output tile
// with tcgen05.mma.cta_group::2 (M=256, N=256, K=16).  CTA r of the pair
// loads rows [128 r, 128 r + 128) of the tile's A and rows [128 r, 128 r +
// 128) of its B (weight) tile into its own shared memory, and holds its 128
// rows of the fp32 accumulator in its own TMEM.  Each SM thus streams half
// of B instead of all of it: per 64-wide k-block 64 KB of shared-memory
// traffic (TMA writes + UMMA reads) against 96 KB for a one-SM 128 x 256
// tile, which is what keeps the tensor pipe fed at ~128 bytes per clock.
// The even CTA issues every UMMA and commits to both CTAs' barriers; both
// CTAs' loads of a stage complete on the even CTA's full barrier.  No load
// uses multicast.
//
// The row statistic of RMSNorm spans all width/256 column tiles of a 128-row
// block, which run on different clusters.  The kernel is persistent (one
// CTA per SM, cooperative cluster launch: every CTA resident) and runs its
// tasks in rounds of one pair tile per cluster, in a linear order (task_of)
// that keeps one projection's weight hot in L2 at a time.  Each CTA posts its
// rows' partial sums of squares and bumps the counter of its 128-row block;
// once the counter reaches the group size (the width/256 tiles of that
// block's q or k), every tile adds the partials in a fixed order (the same
// bits on every tile and every run) and normalises.  v tiles and, with
// epi 0, all tiles have no such dependence.
//
// Warp roles (192 threads per CTA): warps 0-3 epilogue (thread = one row of
// the CTA's half tile, TMEM lane), warp 4 TMA producer (6-stage ring of
// 128x64 A and 128x64 B halves, 128-byte swizzle), warp 5 TMEM allocation
// and, in the even CTA, the UMMA issuer (two 256-column TMEM buffers so the
// epilogue of one tile overlaps the main loop of the next).  Every wait,
// including the wait for a group's partials, is bounded.
#include "ptx.cuh"
#include "ps_b200.h"
#include "internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace psb {
namespace proj {

constexpr int kBM = 128;               // rows per CTA (256 per pair tile)
constexpr int kBN = 256;               // columns per pair tile (128 of B per CTA)
constexpr int kBK = 64;
#ifndef PSB_PROJ_STAGES
#define PSB_PROJ_STAGES 6
#endif
constexpr int kStages = PSB_PROJ_STAGES;  // 32 KiB each
constexpr int kAStage = kBM * kBK * 2;        // 16 KiB
constexpr int kBStage = (kBN / 2) * kBK * 2;  // 16 KiB: this CTA's half of B
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

// One task: a 256 x 256 output tile of one projection (one CTA pair).
struct Task {
  bool valid;
  int kind;   // 0 q, 1 k, 2 v (epi 1); 0 (epi 0)
  int rb;     // 256-row block
  int tile;   // column tile within the projection
  int group;  // epi 1, q/k: rb * 2 + kind
};

// Task of cluster c in round r (P clusters): task index r * P + c in one
// linear order - epi 1: every q tile, then every k tile, then every v tile,
// each kind row block by row block (so one kind's weight stays in L2 while
// its tiles run); epi 0: row block by row block.  A q/k group is the ntile_n
// consecutive tiles of one row block and may straddle two rounds.  No wait
// cycle can form: a tile's epilogue waits only for its group, whose tiles sit
// on ntile_n distinct clusters (the host requires P >= ntile_n), and every
// cluster runs its tasks in increasing index order, so by induction on the
// group index every group completes.
__device__ __forceinline__ Task task_of(const ProjArgs& a, int r, int c, int P) {
  Task t{false, 0, 0, 0, 0};
  const int G = a.ntile_n;
  const int64_t idx = static_cast<int64_t>(r) * P + c;
  if (idx >= a.total_tiles) return t;
  const int64_t per_kind = static_cast<int64_t>(a.row_blocks) * G;
  const int kind = a.epi == 1 ? static_cast<int>(idx / per_kind) : 0;
  const int j = static_cast<int>(idx - kind * per_kind);
  t.valid = true;
  t.kind = kind;
  t.rb = j / G;
  t.tile = j - t.rb * G;
  t.group = t.rb * 2 + kind;
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
  const int P = gridDim.x >> 1;  // clusters
  const int c = blockIdx.x >> 1;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int ksteps = a.kdim / kBK;
  int* status = a.status;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  // The even CTA's barrier i, and barrier i of CTA r, as shared::cluster addresses.
  auto lead_bar = [&](int i) { return mapa_shared(bar(i), 0); };
  auto cta_bar = [&](int i, uint32_t r) { return mapa_shared(bar(i), r); };

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kFull + s), 1);   // even CTA: its producer's arrive + both CTAs' bytes
      mbar_init(bar(kEmpty + s), 1);  // the issuer's commit, in each CTA
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kAccFull + b), 1);   // the issuer's commit, in each CTA
      mbar_init(bar(kAccEmpty + b), 8);  // even CTA: the 4 epilogue warps of each CTA
    }
    mbar_init(bar(kDrain), 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any cross-CTA signal
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
        const int row0 = (t.rb * 2 + static_cast<int>(rank)) * kBM;
        const int n0 = t.tile * kBN + static_cast<int>(rank) * (kBN / 2);
        for (int kk = 0; kk < ksteps; ++kk, ++it) {
          const int s = it % kStages;
          if (it >= kStages) {
            ok = mbar_wait(bar(kEmpty + s), ((it / kStages) - 1) & 1u, abort_flag, status, kErrEmpty);
            if (!ok) break;
          }
          // The even CTA's full barrier counts both CTAs' halves of the stage.
          if (leader) mbar_arrive_expect_tx(bar(kFull + s), 2 * (kAStage + kBStage));
          const uint32_t fb = lead_bar(kFull + s);
          const int k0 = kk * kBK;
          if (a.a_mode == 0) {
            tma_load_2d_pair(smem_u32(sA + s * kAStage), &tm_a, fb, k0, row0);
          } else {
            const int src = k0 / a.a_block_k;
            tma_load_3d_pair(smem_u32(sA + s * kAStage), &tm_a, fb, k0 - src * a.a_block_k, row0, src);
          }
          tma_load_2d_pair(smem_u32(sB + s * kBStage), mw, fb, k0, n0);
        }
      }
      // Every copy issued lands before the pair may exit: the even CTA's full
      // barriers count both CTAs' copies (the odd CTA waits at the final
      // cluster barrier until the even CTA has drained them).
      if (leader)
        for (int j = max(0, it - kStages); j < it; ++j)
          drain_wait(bar(kFull + j % kStages), (j / kStages) & 1u, status);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ UMMA issuer (even CTA)
    if (lane == 0 && leader) {
      const uint32_t idesc = idesc_f16(2 * kBM, kBN, !kFp16, false, false);
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
            umma_ss_pair(acc, das + ((32 * j) >> 4), dbs + ((32 * j) >> 4), idesc, (kk | j) != 0 ? 1u : 0u);
          umma_commit_pair(cta_bar(kEmpty + s, 0));
          umma_commit_pair(cta_bar(kEmpty + s, 1));
        }
        if (!ok) break;
        umma_commit_pair(cta_bar(kAccFull + b, 0));
        umma_commit_pair(cta_bar(kAccFull + b, 1));
        ++seq;
      }
      umma_commit_pair(cta_bar(kDrain, 0));
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
      const int rb128 = t.rb * 2 + static_cast<int>(rank);  // this CTA's 128-row block
      const int m = rb128 * kBM + row;                      // GEMM row
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
          const int group = rb128 * 2 + t.kind;  // the 128-row block's q or k group
          float* part = a.ss_part + static_cast<int64_t>(group) * G * kBM;
          part[t.tile * kBM + row] = ss;
          __threadfence();  // every writer's partial is visible GPU-wide before the group counter moves
          named_bar_sync(1, 128);
          // One thread posts this tile and waits until all G tiles of the
          // group have posted (bounded), then every thread sums the G
          // partials of its row in tile order.
          if (threadIdx.x == 0) {
            __threadfence();
            red_release_gpu_add(a.counters + group, 1u);
            const uint64_t t0 = globaltimer();
            bool waited = true;
            while (ld_acquire_gpu(a.counters + group) < static_cast<unsigned>(G)) {
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
      if (lane == 0) mbar_arrive_cluster(lead_bar(kAccEmpty + b));
    }
  }

  // Both CTAs' UMMAs, copies and TMEM reads are complete before either CTA
  // frees TMEM or exits (the even CTA's UMMAs read the odd CTA's shared
  // memory and write its TMEM).
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
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

template <bool kFp16>
cudaLaunchConfig_t proj_config(int clusters, cudaStream_t stream, cudaLaunchAttribute (&attrs)[2]) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(proj::kThreads);
  cfg.dynamicSmemBytes = proj::kSmemBytes;
  cfg.stream = stream;
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeCooperative;
  attrs[1].val.cooperative = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  return cfg;
}
}  // namespace

// CTA pairs the device keeps resident at once (the persistent grid), queried
// once per device and dtype; 0 on error (with the error recorded).
int proj_clusters(bool fp16) {
  static int cached[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  int& slot = cached[dev][fp16 ? 1 : 0];
  if (slot > 0) return slot;
  if ((fp16 ? prepare_proj<true>() : prepare_proj<false>()) != 0) return 0;
  cudaLaunchAttribute attrs[2];
  cudaLaunchConfig_t cfg = fp16 ? proj_config<true>(1, nullptr, attrs) : proj_config<false>(1, nullptr, attrs);
  cfg.numAttrs = 1;  // the occupancy query takes the cluster shape only
  int n = 0;
  const cudaError_t err = fp16 ? cudaOccupancyMaxActiveClusters(&n, proj::proj_kernel<true>, &cfg)
                               : cudaOccupancyMaxActiveClusters(&n, proj::proj_kernel<false>, &cfg);
  if (err != cudaSuccess || n <= 0) {
    set_cuda_error("projection: cudaOccupancyMaxActiveClusters", err != cudaSuccess ? err : cudaErrorInvalidValue);
    return 0;
  }
  slot = n;
  return n;
}

int launch_proj(const CUtensorMap& ta, const CUtensorMap& tw0, const CUtensorMap& tw1, const CUtensorMap& tw2,
                const ProjArgs& args, bool fp16, int clusters, cudaStream_t stream) {
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
  cudaLaunchAttribute attrs[2];
  cudaError_t err;
  if (fp16) {
    if (int rc = prepare_proj<true>()) return rc;
    const cudaLaunchConfig_t cfg = proj_config<true>(clusters, stream, attrs);
    err = cudaLaunchKernelEx(&cfg, proj_kernel<true>, ta, tw0, tw1, tw2, args);
  } else {
    if (int rc = prepare_proj<false>()) return rc;
    const cudaLaunchConfig_t cfg = proj_config<false>(clusters, stream, attrs);
    err = cudaLaunchKernelEx(&cfg, proj_kernel<false>, ta, tw0, tw1, tw2, args);
  }
  if (err != cudaSuccess) return set_cuda_error("projection launch", err);
  count_launch();
  return 0;
}

}  // namespace psb
