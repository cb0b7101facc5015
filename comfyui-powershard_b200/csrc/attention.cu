// Dense non-causal attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// One CTA computes two 128-row query tiles of one head against every key of
// the sequence.  Keys arrive in 128-row tiles; a "sequence" may be split into
// equal segments (the Ulysses receive buffer holds one segment per source
// rank, each with `seg_rows` rows of which the tail of the last non-empty
// segment is padding), so a tile never straddles two segments and the last
// tile of a segment is masked to the segment's valid rows.
//
// Warp roles (320 threads):
//   warps 0-3  softmax + epilogue of query tile 0 (thread = one query row)
//   warps 4-7  softmax + epilogue of query tile 1
//   warp  8    TMA producer: Q tiles once, then K_i, V_i into a 4-stage ring
//   warp  9    TMEM allocator and UMMA issuer (one elected lane)
// 10 warps put 3 warps on two of the four SM sub-partitions, which caps a
// thread at 168 registers; the softmax path is arranged to fit that (the S
// row is dead before the rare O rescale loads O).
//
// TMEM (512 columns x 128 lanes, fp32):
//   [  0,128) S0 = Q0 K^T   (P0, bf16/fp16 pairs, overwrites columns [0,64))
//   [128,256) S1 = Q1 K^T   (P1 overwrites [128,192))
//   [256,384) O0 accumulator,  [384,512) O1 accumulator
//
// UMMA issue order per key tile i (one thread, in-order tensor pipe):
//   S0_i = Q0 K_i^T,  O1 += P1_{i-1} V_{i-1},  S1_i = Q1 K_i^T,  O0 += P0_i V_i
// so while one softmax warpgroup exponentiates, the tensor pipe works on the
// other tile.  A tcgen05.commit tracks every earlier UMMA of the issuing
// thread, hence "S_t full" also means the previous O_t update is complete and
// the softmax warps may rescale O_t in place.
//
// Online softmax in the log2 domain with a lazily updated row maximum: the
// running max m is only raised (and O, l rescaled) when a tile's max exceeds
// it by more than 8, so P <= 2^8 and rescales are rare after the first tiles.
#include "ptx.cuh"
#include "internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace psb {
namespace attn {

constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kHeadDim = 128;
constexpr int kStages = 4;
constexpr int kTileBytes = kBlockN * kHeadDim * 2;  // 32 KiB: one Q, K or V tile
constexpr int kHalfTile = kTileBytes / 2;           // one 64-column SW128 half
constexpr int kThreads = 320;
constexpr int kSmemQ = 2 * kTileBytes;
constexpr int kSmemKV = kStages * kTileBytes;
constexpr int kSmemBarOff = kSmemQ + kSmemKV;

enum Bar : int {
  kBarQ = 0,
  kBarFull = 1,
  kBarEmpty = kBarFull + kStages,
  kBarS = kBarEmpty + kStages,
  kBarP = kBarS + 2,
  kBarO = kBarP + 2,
  kBarDrain = kBarO + 1,
  kNumBars
};
constexpr int kSmemBytes = kSmemBarOff + 256 + 1024;  // barriers + TMEM slot + 1 KiB align slack
static_assert(kNumBars * 8 + 8 <= 256, "barrier block overflow");

// Device status codes written on a bounded-wait timeout (first error wins).
enum Err : int {
  kErrQ = 101,
  kErrEmpty = 102,
  kErrFull = 103,
  kErrP = 104,
  kErrS = 105,
  kErrO = 106,
  kErrDrain = 107,
};

__device__ __forceinline__ void tile_coord(int t, int full_segs, int tiles_per_seg, int seg_rows,
                                           int len, int& seg, int& row0, int& valid) {
  if (t < full_segs * tiles_per_seg) {
    seg = t / tiles_per_seg;
    row0 = (t - seg * tiles_per_seg) * kBlockM;
    valid = min(kBlockM, seg_rows - row0);
  } else {
    seg = full_segs;
    row0 = (t - full_segs * tiles_per_seg) * kBlockM;
    valid = min(kBlockM, len - full_segs * seg_rows - row0);
  }
}

// Bounded wait whose outcome is uniform across the warp (a lane that timed
// out drags the whole warp out, so .sync.aligned tcgen05 ops stay converged).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, int code) {
  bool ok = mbar_wait(bar, parity, abort_flag, status, code);
  return __all_sync(0xffffffffu, ok);
}

// Wait used only while tearing down: ignores the abort flag (copies/UMMAs in
// flight must land before shared memory / TMEM is released) but is bounded.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, int* status) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      if (status) atomicCAS(status, 0, kErrDrain);
      return;
    }
  }
}

template <bool kFp16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return kFp16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
}

template <bool kFp16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + kSmemQ;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int batch = blockIdx.z;
  const int kv_head = head / args.group;
  const int tq0 = blockIdx.x * 2;
  const int tq1 = tq0 + 1;
  const int T = args.num_kv_tiles;
  int* status = args.status;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(bar(kBarQ), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarFull + s), 1);
      mbar_init(bar(kBarEmpty + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kBarS + t), 1);
      mbar_init(bar(kBarP + t), 128);
    }
    mbar_init(bar(kBarO), 1);
    mbar_init(bar(kBarDrain), 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int sg0, r00, v0, sg1, r01, v1;
      tile_coord(tq0, args.q_full_segs, args.q_tiles_per_seg, args.seg_rows_q, args.len_q, sg0, r00, v0);
      if (tq1 < args.num_q_tiles) {
        tile_coord(tq1, args.q_full_segs, args.q_tiles_per_seg, args.seg_rows_q, args.len_q, sg1, r01, v1);
      } else {  // no second tile: recompute tile 0, never stored
        sg1 = sg0;
        r01 = r00;
      }
      mbar_arrive_expect_tx(bar(kBarQ), 2 * kTileBytes);
      for (int c = 0; c < 2; ++c) {
        tma_load_5d(smem_u32(sQ + c * kHalfTile), &tm_q, bar(kBarQ), c * 64, head, r00, sg0, batch);
        tma_load_5d(smem_u32(sQ + kTileBytes + c * kHalfTile), &tm_q, bar(kBarQ), c * 64, head, r01,
                    sg1, batch);
      }
      uint32_t load = 0;
      bool ok = true;
      for (int i = 0; i < T && ok; ++i) {
        int seg, row0, valid;
        tile_coord(i, args.kv_full_segs, args.kv_tiles_per_seg, args.seg_rows_k, args.len_k, seg, row0,
                   valid);
        for (int kv = 0; kv < 2; ++kv) {
          const int stage = load % kStages;
          const uint32_t phase = (load / kStages) & 1u;
          ok = mbar_wait(bar(kBarEmpty + stage), phase ^ 1u, abort_flag, status, kErrEmpty);
          if (!ok) break;
          mbar_arrive_expect_tx(bar(kBarFull + stage), kTileBytes);
          const CUtensorMap* map = kv ? &tm_v : &tm_k;
          uint8_t* dst = sKV + stage * kTileBytes;
          tma_load_5d(smem_u32(dst), map, bar(kBarFull + stage), 0, kv_head, row0, seg, batch);
          tma_load_5d(smem_u32(dst + kHalfTile), map, bar(kBarFull + stage), 64, kv_head, row0, seg,
                      batch);
          ++load;
        }
      }
      // Every copy issued must land before the CTA may exit.
      drain_wait(bar(kBarQ), 0, status);
      const uint32_t first = load > kStages ? load - kStages : 0;
      for (uint32_t j = first; j < load; ++j)
        drain_wait(bar(kBarFull + (j % kStages)), (j / kStages) & 1u, status);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(kBlockM, kBlockN, !kFp16, false, false);
      const uint32_t id_pv = idesc_f16(kBlockM, kHeadDim, !kFp16, false, true);
      const uint32_t sq0 = smem_u32(sQ), sq1 = smem_u32(sQ + kTileBytes);
      const uint32_t skv = smem_u32(sKV);
      auto mma_s = [&](int t, int stage) {
        const uint32_t qa = t ? sq1 : sq0;
        const uint32_t kb = skv + stage * kTileBytes;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t off = (s >> 2) * kHalfTile + (s & 3) * 32;
          umma_ss(tmem + 128 * t, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(kb + off, 16, 1024), id_qk,
                  s > 0);
        }
      };
      auto mma_pv = [&](int t, int stage, bool accumulate) {
        const uint32_t vb = skv + stage * kTileBytes;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          umma_ts(tmem + 256 + 128 * t, tmem + 128 * t + s * 8, sdesc_sw128(vb + s * 2048, kHalfTile, 1024),
                  id_pv, (accumulate || s > 0) ? 1u : 0u);
        }
      };
      auto stage_of = [](uint32_t load) { return static_cast<int>(load % kStages); };
      auto phase_of = [](uint32_t load) { return (load / kStages) & 1u; };

      bool ok = mbar_wait(bar(kBarQ), 0, abort_flag, status, kErrQ);
      int prev_v = 0;
      for (int i = 0; i < T && ok; ++i) {
        const uint32_t lk = 2u * i, lv = 2u * i + 1u;
        ok = mbar_wait(bar(kBarFull + stage_of(lk)), phase_of(lk), abort_flag, status, kErrFull);
        if (!ok) break;
        tc_fence_after();
        mma_s(0, stage_of(lk));
        umma_commit(bar(kBarS + 0));
        if (i > 0) {
          ok = mbar_wait(bar(kBarP + 1), (i - 1) & 1u, abort_flag, status, kErrP);
          if (!ok) break;
          tc_fence_after();
          mma_pv(1, prev_v, i > 1);
          umma_commit(bar(kBarEmpty + prev_v));
        }
        mma_s(1, stage_of(lk));
        umma_commit(bar(kBarS + 1));
        umma_commit(bar(kBarEmpty + stage_of(lk)));
        ok = mbar_wait(bar(kBarFull + stage_of(lv)), phase_of(lv), abort_flag, status, kErrFull);
        if (ok) ok = mbar_wait(bar(kBarP + 0), i & 1u, abort_flag, status, kErrP);
        if (!ok) break;
        tc_fence_after();
        mma_pv(0, stage_of(lv), i > 0);
        prev_v = stage_of(lv);
      }
      if (ok) {
        ok = mbar_wait(bar(kBarP + 1), (T - 1) & 1u, abort_flag, status, kErrP);
        if (ok) {
          tc_fence_after();
          mma_pv(1, prev_v, T > 1);
          umma_commit(bar(kBarEmpty + prev_v));
          umma_commit(bar(kBarO));
        }
      }
      // All issued UMMAs complete before TMEM is released.
      umma_commit(bar(kBarDrain));
      drain_wait(bar(kBarDrain), 0, status);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + 128 * t;
    const uint32_t o_addr = tmem + lane_off + 256 + 128 * t;
    const float scale_log2 = args.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < T; ++i) {
      int seg, row0, valid;
      tile_coord(i, args.kv_full_segs, args.kv_tiles_per_seg, args.seg_rows_k, args.len_k, seg, row0,
                 valid);
      ok = warp_wait(bar(kBarS + t), i & 1u, abort_flag, status, kErrS);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld32_at<0>(s_addr + 0, sr);
      tmem_ld32_at<32>(s_addr + 32, sr);
      tmem_ld32_at<64>(s_addr + 64, sr);
      tmem_ld32_at<96>(s_addr + 96, sr);
      tmem_wait_ld();
      float s[128];
#pragma unroll
      for (int j = 0; j < 128; ++j) s[j] = __uint_as_float(sr[j]);
      if (valid < kBlockN) {
#pragma unroll
        for (int j = 0; j < 128; ++j)
          if (j >= valid) s[j] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int j = 4; j < 128; j += 4) {
        mx0 = fmaxf(mx0, s[j]);
        mx1 = fmaxf(mx1, s[j + 1]);
        mx2 = fmaxf(mx2, s[j + 2]);
        mx3 = fmaxf(mx3, s[j + 3]);
      }
      const float m_tile = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * scale_log2;
      // Raise the running max (warp-uniformly) only when it grew by > 8.
      float alpha = 1.f;
      bool rescale = false;
      if (i == 0) {
        m = m_tile;
      } else if (__any_sync(0xffffffffu, m_tile - m > 8.f)) {
        const float m_new = fmaxf(m, m_tile);
        alpha = ex2_approx(m - m_new);
        m = m_new;
        rescale = true;
      }
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float p0 = ex2_approx(fmaf(s[32 * c + 2 * j], scale_log2, -m));
          const float p1 = ex2_approx(fmaf(s[32 * c + 2 * j + 1], scale_log2, -m));
          sum0 += p0;
          sum1 += p1;
          pk[j] = pack2<kFp16>(p0, p1);
        }
        tmem_st16(s_addr + 16 * c, pk);
      }
      l = fmaf(l, alpha, sum0 + sum1);
      if (rescale) {  // O_t is idle here: its last update completed before S_t was signalled
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
          tmem_st32(o_addr + 32 * c, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarP + t));
    }
    if (ok) ok = warp_wait(bar(kBarO), 0, abort_flag, status, kErrO);
    tc_fence_after();
    if (ok) {
      const int tq = t ? tq1 : tq0;
      int seg = 0, row0 = 0, valid = 0;
      if (tq < args.num_q_tiles)
        tile_coord(tq, args.q_full_segs, args.q_tiles_per_seg, args.seg_rows_q, args.len_q, seg, row0, valid);
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      const bool store = row < valid;
      const int64_t oidx = batch * args.o_stride[0] + seg * args.o_stride[1] +
                           static_cast<int64_t>(row0 + row) * args.o_stride[2] + head * args.o_stride[3];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(o_addr + 32 * c, o);
        tmem_wait_ld();
        if (store) {
          if (args.out_fp32) {
            float4* orow = reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + oidx + 32 * c);
#pragma unroll
            for (int u = 0; u < 8; ++u)
              orow[u] = make_float4(__uint_as_float(o[4 * u + 0]) * inv_l, __uint_as_float(o[4 * u + 1]) * inv_l,
                                    __uint_as_float(o[4 * u + 2]) * inv_l, __uint_as_float(o[4 * u + 3]) * inv_l);
          } else {
            uint16_t* orow = reinterpret_cast<uint16_t*>(args.out) + oidx + 32 * c;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint4 v;
              v.x = pack2<kFp16>(__uint_as_float(o[8 * u + 0]) * inv_l, __uint_as_float(o[8 * u + 1]) * inv_l);
              v.y = pack2<kFp16>(__uint_as_float(o[8 * u + 2]) * inv_l, __uint_as_float(o[8 * u + 3]) * inv_l);
              v.z = pack2<kFp16>(__uint_as_float(o[8 * u + 4]) * inv_l, __uint_as_float(o[8 * u + 5]) * inv_l);
              v.w = pack2<kFp16>(__uint_as_float(o[8 * u + 6]) * inv_l, __uint_as_float(o[8 * u + 7]) * inv_l);
              *reinterpret_cast<uint4*>(orow + 8 * u) = v;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn

namespace {
template <bool kFp16>
int prepare_kernel() {
  const cudaError_t err = cudaFuncSetAttribute(attn::attn_fwd_kernel<kFp16>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, attn::kSmemBytes);
  return err == cudaSuccess ? 0 : set_cuda_error("attention: cudaFuncSetAttribute", err);
}
}  // namespace

int launch_attention(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                     const AttnArgs& args, int heads_q, int batch, bool fp16, cudaStream_t stream) {
  using namespace attn;
  const dim3 grid((args.num_q_tiles + 1) / 2, heads_q, batch);
  const dim3 block(kThreads);
  if (fp16) {
    if (int rc = prepare_kernel<true>()) return rc;
    attn_fwd_kernel<true><<<grid, block, kSmemBytes, stream>>>(tq, tk, tv, args);
  } else {
    if (int rc = prepare_kernel<false>()) return rc;
    attn_fwd_kernel<false><<<grid, block, kSmemBytes, stream>>>(tq, tk, tv, args);
  }
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_cuda_error("attention launch", err);
  return 0;
}

}  // namespace psb
