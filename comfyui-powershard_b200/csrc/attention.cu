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
//   warp  8    TMA producer: Q tiles once, then K_i / V_i into 2-stage rings
//   warp  9    TMEM allocator and UMMA issuer (one lane)
// 10 warps put 3 warps on two of the four SM sub-partitions, which caps a
// thread at 168 registers; the softmax fits that.
//
// TMEM (512 columns x 128 lanes, fp32):
//   [  0,128) S0 = Q0 K^T   (P0, bf16/fp16 pairs, overwrites columns [0,64))
//   [128,256) S1 = Q1 K^T   (P1 overwrites [128,192))
//   [256,384) O0 accumulator,  [384,512) O1 accumulator
//
// UMMA issue order per key tile i (one thread, in-order tensor pipe):
//   S0_i = Q0 K_i^T,  O1 += P1_{i-1} V_{i-1},  S1_i = Q1 K_i^T,  O0 += P0_i V_i
// so while one softmax warpgroup exponentiates, the tensor pipe works on the
// other tile, and S_t,i+1 is always issued after the PV that reads P_t,i.
// A tcgen05.commit tracks every earlier UMMA of the issuing thread, so only
// two commits per tile are needed: "S_t full" also means O_t's previous update
// is complete (the softmax warps may rescale O_t in place), and S1_i complete
// means K_i and V_{i-1} are free (relayed to the producer by a softmax-1
// thread).  An issuing thread spends ~50 cycles per tcgen05.mma (measured),
// so the issuer does nothing but wait and issue.
//
// Online softmax in the log2 domain with a lazily updated row maximum: the
// running max m is only raised (and O, l rescaled) when a tile's max exceeds
// it by more than 8, so P <= 2^8.  P_t is released to the PV UMMAs in two
// 64-key parts, so the tensor pipe starts on the first half while the softmax
// writes the second.  The exponentials use ex2.approx on the MUFU; measured on
// B200, moving part of them to an FMA-pipe polynomial or fusing the row max
// into the exponential pass made the softmax slower.
#include "ptx.cuh"
#include "ps_b200.h"
#include "internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace psb {
namespace attn {

constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kHeadDim = 128;
constexpr int kKStages = 2;                          // K ring
constexpr int kVStages = 2;                          // V ring
constexpr int kTileBytes = kBlockN * kHeadDim * 2;   // 32 KiB: one Q, K or V tile
constexpr int kHalfTile = kTileBytes / 2;            // one 64-column SW128 half
constexpr int kThreads = 320;                        // 10 warps
constexpr int kSmemQ = 2 * kTileBytes;
constexpr int kSmemK = kKStages * kTileBytes;
constexpr int kSmemV = kVStages * kTileBytes;
constexpr int kSmemBarOff = kSmemQ + kSmemK + kSmemV;
// P_t is released to the PV UMMAs in kPParts parts of 128/kPParts keys, so
// the tensor pipe starts on the first keys while the softmax writes the rest.
#ifndef PSB_P_PARTS
#define PSB_P_PARTS 2
#endif
constexpr int kPParts = PSB_P_PARTS;
static_assert(kPParts == 1 || kPParts == 2 || kPParts == 4, "P parts: 1, 2 or 4");
constexpr int kChunksPerPart = 4 / kPParts;  // 32-key chunks per part

enum Bar : int {
  kBarQ = 0,
  kBarKFull = 1,
  kBarVFull = kBarKFull + kKStages,
  kBarS = kBarVFull + kVStages,  // [2] S_t,i computed (issuer commit)
  kBarFree = kBarS + 2,          // [2] FREE[i%2]: S1_i observed complete -> K_i, V_{i-1} free
  kBarP = kBarFree + 2,          // [2] P_t written (128 softmax threads)
  kBarPH = kBarP + 2,            // [2][kPParts-1] leading parts of P_t written
  kBarO = kBarPH + 2 * (kPParts - 1),  // O_0 and O_1 final
  kBarDrain = kBarO + 1,         // every UMMA of the issuer complete
  kNumBars = kBarDrain + 1
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

// Walks the key tiles - the prefix range first, then the segmented range
// segment by segment (skipping empty segments) - returning each tile's
// segment, first row and valid rows, without divisions.
struct KeyCursor {
  int i = 0, seg = 0, row0 = 0;
  // Position the cursor so that the next call of next() returns tile n.
  __device__ __forceinline__ void skip(const AttnArgs& a, int n) {
    const int take = min(n, max(a.pre_tiles - i, 0));
    i += take;
    n -= take;
    while (n > 0) {
      while (row0 >= a.valid_k[seg] && seg + 1 < a.nsegs_k) {
        ++seg;
        row0 = 0;
      }
      const int left = (a.valid_k[seg] - row0 + kBlockN - 1) / kBlockN;
      if (left <= 0) break;
      const int t = min(n, left);
      row0 += t * kBlockN;
      i += t;
      n -= t;
    }
  }
  __device__ __forceinline__ void next(const AttnArgs& a, bool& prefix, int& s, int& r, int& valid) {
    if (i < a.pre_tiles) {
      prefix = true;
      s = 0;
      r = i * kBlockN;
      valid = min(kBlockN, a.pre_len - r);
      ++i;
      return;
    }
    ++i;
    prefix = false;
    while (row0 >= a.valid_k[seg] && seg + 1 < a.nsegs_k) {
      ++seg;
      row0 = 0;
    }
    s = seg;
    r = row0;
    valid = min(kBlockN, a.valid_k[seg] - row0);
    row0 += kBlockN;
  }
};

// Query tile t: prefix tiles first, then q_tiles_per_seg tiles per segment
// (a tile past its segment's valid rows has valid <= 0 and is never stored).
__device__ __forceinline__ void q_tile(const AttnArgs& a, int t, bool& prefix, int& seg, int& row0, int& valid) {
  if (t < a.pre_tiles) {
    prefix = true;
    seg = 0;
    row0 = t * kBlockM;
    valid = min(kBlockM, a.pre_len - row0);
  } else {
    prefix = false;
    const int u = t - a.pre_tiles;
    seg = u / a.q_tiles_per_seg;
    row0 = (u - seg * a.q_tiles_per_seg) * kBlockM;
    valid = min(kBlockM, a.valid_q[seg] - row0);
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

__device__ __forceinline__ float row_max128(const float (&s)[128]) {
  float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
  for (int j = 0; j < 128; j += 8) {
    mx0 = fmax3(mx0, s[j], s[j + 1]);
    mx1 = fmax3(mx1, s[j + 2], s[j + 3]);
    mx2 = fmax3(mx2, s[j + 4], s[j + 5]);
    mx3 = fmax3(mx3, s[j + 6], s[j + 7]);
  }
  return fmaxf(fmax3(mx0, mx1, mx2), mx3);
}

template <bool kFp16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_qp,
                    const __grid_constant__ CUtensorMap tm_kp, const __grid_constant__ CUtensorMap tm_vp,
                    const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kSmemQ;
  uint8_t* sV = sK + kSmemK;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Work unit and key range of this CTA.
  const int bx = blockIdx.x;
  const bool partial = bx >= args.full_units;
  const int nparts = partial ? args.split : 1;
  const int v_split = partial ? bx - args.full_units : 0;
  const int unit = partial ? args.full_units + v_split / args.split : bx;
  const int part = partial ? v_split - (v_split / args.split) * args.split : 0;
  const int slot = partial ? v_split : 0;
  const int pair = unit % args.npairs;
  const int head = (unit / args.npairs) % args.grid_heads;
  const int batch = unit / args.npairs / args.grid_heads;
  const int kv_head = head / args.group;
  const int tq0 = pair * 2;
  const int tq1 = tq0 + 1;
  const int k_begin = part * args.num_kv_tiles / nparts;
  const int T = (part + 1) * args.num_kv_tiles / nparts - k_begin;
  int* status = args.status;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(bar(kBarQ), 1);
    for (int s = 0; s < kKStages; ++s) mbar_init(bar(kBarKFull + s), 1);
    for (int s = 0; s < kVStages; ++s) mbar_init(bar(kBarVFull + s), 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kBarS + t), 1);
      mbar_init(bar(kBarFree + t), 1);
      mbar_init(bar(kBarP + t), 128);
      for (int q = 0; q + 1 < kPParts; ++q) mbar_init(bar(kBarPH + t * (kPParts - 1) + q), 128);
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
      bool p0, p1;
      int sg0, r00, v0, sg1, r01, v1;
      q_tile(args, tq0, p0, sg0, r00, v0);
      if (tq1 < args.num_q_tiles) {
        q_tile(args, tq1, p1, sg1, r01, v1);
      } else {  // no second tile: recompute tile 0, never stored
        p1 = p0;
        sg1 = sg0;
        r01 = r00;
      }
      mbar_arrive_expect_tx(bar(kBarQ), 2 * kTileBytes);
      for (int c = 0; c < 2; ++c) {
        tma_load_5d(smem_u32(sQ + c * kHalfTile), p0 ? &tm_qp : &tm_q, bar(kBarQ), c * 64, head, r00, sg0, batch);
        tma_load_5d(smem_u32(sQ + kTileBytes + c * kHalfTile), p1 ? &tm_qp : &tm_q, bar(kBarQ), c * 64, head, r01,
                    sg1, batch);
      }
      // Stage reuse.  The issuer commits S_1,i after S0_i, PV1_{i-1} and S1_i,
      // so once S1_i is complete K_i and V_{i-1} are no longer read; a
      // softmax-1 thread then arrives on FREE[i%2].  K_j reuses K_{j-2}'s
      // stage (signal j-2); V_j reuses V_{j-2}'s stage (signal j-1).  FREE[s]
      // cannot complete another phase before the producer has loaded the K
      // tile gated on it, so parity waits never alias.
      KeyCursor cur;
      cur.skip(args, k_begin);
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < T && ok; ++i) {
        bool pre;
        int seg, row0, valid;
        cur.next(args, pre, seg, row0, valid);
        const CUtensorMap* mk = pre ? &tm_kp : &tm_k;
        const CUtensorMap* mv = pre ? &tm_vp : &tm_v;
        const int st = i % kKStages;
        if (i >= kKStages) {
          ok = mbar_wait(bar(kBarFree + (i & 1)), ((i - 2) >> 1) & 1u, abort_flag, status, kErrEmpty);
          if (!ok) break;
        }
        mbar_arrive_expect_tx(bar(kBarKFull + st), kTileBytes);
        tma_load_5d(smem_u32(sK + st * kTileBytes), mk, bar(kBarKFull + st), 0, kv_head, row0, seg, batch);
        tma_load_5d(smem_u32(sK + st * kTileBytes + kHalfTile), mk, bar(kBarKFull + st), 64, kv_head, row0, seg,
                    batch);
        issued = 2 * i + 1;
        if (i >= kVStages) {
          ok = mbar_wait(bar(kBarFree + ((i - 1) & 1)), ((i - 1) >> 1) & 1u, abort_flag, status, kErrEmpty);
          if (!ok) break;
        }
        mbar_arrive_expect_tx(bar(kBarVFull + st), kTileBytes);
        tma_load_5d(smem_u32(sV + st * kTileBytes), mv, bar(kBarVFull + st), 0, kv_head, row0, seg, batch);
        tma_load_5d(smem_u32(sV + st * kTileBytes + kHalfTile), mv, bar(kBarVFull + st), 64, kv_head, row0, seg,
                    batch);
        issued = 2 * i + 2;
      }
      // Every copy issued must land before the CTA may exit.
      drain_wait(bar(kBarQ), 0, status);
      const int kv_issued = (issued + 1) / 2;  // key tiles with at least the K copy issued
      for (int i = max(0, kv_issued - kKStages); i < kv_issued; ++i) {
        const int st = i % kKStages;
        const uint32_t ph = (i / kKStages) & 1u;
        drain_wait(bar(kBarKFull + st), ph, status);
        if (2 * i + 2 <= issued) drain_wait(bar(kBarVFull + st), ph, status);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ UMMA issuer (one lane)
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(kBlockM, kBlockN, !kFp16, false, false);
      const uint32_t id_pv = idesc_f16(kBlockM, kHeadDim, !kFp16, false, true);
      // Descriptor bases; per-UMMA offsets are added to the start-address field
      // (all shared addresses stay below 256 KiB, so the 14-bit field never carries).
      const uint64_t dq0 = sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t dq1 = sdesc_sw128(smem_u32(sQ + kTileBytes), 16, 1024);
      const uint64_t dk = sdesc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t dv = sdesc_sw128(smem_u32(sV), kHalfTile, 1024);
      auto mma_s = [&](int t, int st) {
        const uint64_t dq = t ? dq1 : dq0;
        const uint64_t dks = dk + static_cast<uint64_t>(st * (kTileBytes >> 4));
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t off = ((s >> 2) * kHalfTile + (s & 3) * 32) >> 4;
          umma_ss(tmem + 128 * t, dq + off, dks + off, id_qk, s > 0);
        }
      };
      // O_t (+)= P_t V for the keys of part q (8/kPParts UMMAs of K=16).
      auto mma_pv = [&](int t, int st, int q, bool accumulate) {
        const uint64_t dvs = dv + static_cast<uint64_t>(st * (kTileBytes >> 4));
#pragma unroll
        for (int k = 0; k < 8 / kPParts; ++k) {
          const int s = (8 / kPParts) * q + k;
          umma_ts(tmem + 256 + 128 * t, tmem + 128 * t + s * 8, dvs + ((s * 2048) >> 4), id_pv,
                  (accumulate || s > 0) ? 1u : 0u);
        }
      };
      // P_t arrives in parts; each part's UMMAs are issued as soon as it is written.
      auto pv_both = [&](int t, int st, uint32_t parity, bool accumulate) -> bool {
#pragma unroll
        for (int q = 0; q < kPParts; ++q) {
          const int b = q + 1 < kPParts ? kBarPH + t * (kPParts - 1) + q : kBarP + t;
          if (!mbar_wait(bar(b), parity, abort_flag, status, kErrP)) return false;
          tc_fence_after();
          mma_pv(t, st, q, accumulate);
        }
        return true;
      };
      // Issue order per key tile i: S0_i, PV1_{i-1}, S1_i, PV0_i.
      bool ok = mbar_wait(bar(kBarQ), 0, abort_flag, status, kErrQ);
      for (int i = 0; i < T && ok; ++i) {
        const int st = i % kKStages;
        const uint32_t ph = (i / kKStages) & 1u;
        ok = mbar_wait(bar(kBarKFull + st), ph, abort_flag, status, kErrFull);
        if (!ok) break;
        tc_fence_after();
        mma_s(0, st);
        umma_commit(bar(kBarS + 0));
        if (i > 0) {
          ok = pv_both(1, (i - 1) % kVStages, (i - 1) & 1u, i > 1);
          if (!ok) break;
        }
        mma_s(1, st);
        umma_commit(bar(kBarS + 1));
        ok = mbar_wait(bar(kBarVFull + st), ph, abort_flag, status, kErrFull);
        if (ok) ok = pv_both(0, st, i & 1u, i > 0);
        if (!ok) break;
      }
      if (ok) {
        ok = pv_both(1, (T - 1) % kVStages, (T - 1) & 1u, T > 1);
        if (ok) umma_commit(bar(kBarO));
      }
      // All issued UMMAs complete before TMEM is released.
      umma_commit(bar(kBarDrain));
      drain_wait(bar(kBarDrain), 0, status);
    }
  } else if (warp < 8) {
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
    KeyCursor cur;
    cur.skip(args, k_begin);
    for (int i = 0; i < T; ++i) {
      bool pre_unused;
      int seg_unused, row_unused, valid;
      cur.next(args, pre_unused, seg_unused, row_unused, valid);
      ok = warp_wait(bar(kBarS + t), i & 1u, abort_flag, status, kErrS);
      if (!ok) break;
      if (t == 1 && threadIdx.x == 128) mbar_arrive(bar(kBarFree + (i & 1)));
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
      const bool masked = valid < kBlockN;
      if (masked) {
#pragma unroll
        for (int j = 0; j < 128; ++j)
          if (j >= valid) s[j] = -INFINITY;
      }
      float alpha = 1.f, sum;
      bool rescale = false;
      // Row max first (lazy running max: raised warp-uniformly only when it
      // grew by > 8), then the exponentials.
      const float m_tile = row_max128(s) * scale_log2;
      if (i == 0) {
        m = m_tile;
      } else if (__any_sync(0xffffffffu, m_tile - m > 8.f)) {
        const float m_new = fmaxf(m, m_tile);
        alpha = ex2_approx(m - m_new);
        m = m_new;
        rescale = true;
      }
      {
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
          if (c == (kPParts > 1 ? kChunksPerPart - 1 : 3)) {
            // The rare O rescale goes here, before the first PV part of this
            // tile is released (O_t's last update completed before S_t was
            // signalled); the row's first chunks are dead by now.
            if (rescale) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint32_t o[32];
                tmem_ld32(o_addr + 32 * q, o);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
                tmem_st32(o_addr + 32 * q, o);
              }
            }
          }
          if ((c + 1) % kChunksPerPart == 0 && c < 3) {  // part (c+1)/kChunksPerPart - 1 written
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(kBarPH + t * (kPParts - 1) + (c + 1) / kChunksPerPart - 1));
          }
        }
        sum = sum0 + sum1;
      }
      l = fmaf(l, alpha, sum);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(kBarP + t));
    }
    if (ok) ok = warp_wait(bar(kBarO), 0, abort_flag, status, kErrO);
    tc_fence_after();
    const int tq = t ? tq1 : tq0;
    bool pre = false;
    int seg = 0, row0 = 0, valid = 0;
    if (tq < args.num_q_tiles) q_tile(args, tq, pre, seg, row0, valid);
    const float inv_l = l > 0.f ? 1.f / l : 0.f;
    void* const obase = pre ? args.pre_out : args.seg_out[seg];
    const int64_t* ost = pre ? args.pre_o_stride : args.o_stride;
    const int64_t otile = batch * ost[0] + static_cast<int64_t>(row0) * ost[2] + head * ost[3];
    if (partial) {
      // One part of a split key range: O / l in fp32 and m + log2(l), merged
      // by attn_combine_kernel (tcgen05.ld stays warp-collective).
      if (ok) {
        float* wrow = args.ws_o + ((static_cast<int64_t>(slot) * 2 + t) * kBlockM + row) * kHeadDim;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + 32 * c, o);
          tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(wrow + 32 * c);
#pragma unroll
          for (int u = 0; u < 8; ++u)
            dst[u] = make_float4(__uint_as_float(o[4 * u + 0]) * inv_l, __uint_as_float(o[4 * u + 1]) * inv_l,
                                 __uint_as_float(o[4 * u + 2]) * inv_l, __uint_as_float(o[4 * u + 3]) * inv_l);
        }
        args.ws_lse[(slot * 2 + t) * kBlockM + row] = l > 0.f ? m + __log2f(l) : -INFINITY;
      }
    } else if (args.out_fp32) {
      // tcgen05.ld is warp-collective: every lane loads, only valid rows store.
      if (ok) {
        float* orow = reinterpret_cast<float*>(obase) + otile + static_cast<int64_t>(row) * ost[2];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + 32 * c, o);
          tmem_wait_ld();
          if (row < valid) {
            float4* dst = reinterpret_cast<float4*>(orow + 32 * c);
#pragma unroll
            for (int u = 0; u < 8; ++u)
              dst[u] = make_float4(__uint_as_float(o[4 * u + 0]) * inv_l, __uint_as_float(o[4 * u + 1]) * inv_l,
                                   __uint_as_float(o[4 * u + 2]) * inv_l, __uint_as_float(o[4 * u + 3]) * inv_l);
          }
        }
      }
    } else {
      // Stage the 16-bit tile in K stage t (idle once every UMMA has
      // completed): row r, 16-byte chunk k at r*256 + ((k ^ (r & 15)) << 4),
      // so both the row-per-thread writes and the row-major reads below touch
      // each bank group once per 128 bytes.  Then 16 threads store each
      // 256-byte output row with consecutive 16-byte stores, which keeps the
      // rows whole when they cross NVLink.
      uint8_t* stage = sK + t * kTileBytes;
      if (ok) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 v;
            v.x = pack2<kFp16>(__uint_as_float(o[8 * u + 0]) * inv_l, __uint_as_float(o[8 * u + 1]) * inv_l);
            v.y = pack2<kFp16>(__uint_as_float(o[8 * u + 2]) * inv_l, __uint_as_float(o[8 * u + 3]) * inv_l);
            v.z = pack2<kFp16>(__uint_as_float(o[8 * u + 4]) * inv_l, __uint_as_float(o[8 * u + 5]) * inv_l);
            v.w = pack2<kFp16>(__uint_as_float(o[8 * u + 6]) * inv_l, __uint_as_float(o[8 * u + 7]) * inv_l);
            const int k = 4 * c + u;
            *reinterpret_cast<uint4*>(stage + row * 256 + ((k ^ (row & 15)) << 4)) = v;
          }
        }
      }
      named_bar_sync(1 + t, 128);  // all 128 threads of the group, whatever their wait outcome
      if (ok) {
        const int sub = threadIdx.x & 127;
        const int k = sub & 15;
        uint16_t* const obase16 = reinterpret_cast<uint16_t*>(obase) + otile + 8 * k;
#pragma unroll 4
        for (int p = 0; p < 16; ++p) {
          const int r = p * 8 + (sub >> 4);
          if (r < valid) {
            const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 256 + ((k ^ (r & 15)) << 4));
            *reinterpret_cast<uint4*>(obase16 + static_cast<int64_t>(r) * ost[2]) = v;
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

// Merges the split parts of the last wave's units: for each valid query row,
// out = sum_p w_p o_p / sum_p w_p with w_p = 2^(lse_p - max lse), the
// log-sum-exp combination of partial softmax results.  One CTA per (unit,
// query tile); 16 threads per row, 8 columns each.
template <bool kFp16>
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs args) {
  const int u = blockIdx.x >> 1;
  const int t = blockIdx.x & 1;
  const int unit = args.full_units + u;
  const int pair = unit % args.npairs;
  const int head = (unit / args.npairs) % args.grid_heads;
  const int batch = unit / args.npairs / args.grid_heads;
  const int tq = pair * 2 + t;
  if (tq >= args.num_q_tiles) return;
  bool pre;
  int seg, row0, valid;
  q_tile(args, tq, pre, seg, row0, valid);
  void* const obase = pre ? args.pre_out : args.seg_out[seg];
  const int64_t* ost = pre ? args.pre_o_stride : args.o_stride;
  const int64_t otile = batch * ost[0] + static_cast<int64_t>(row0) * ost[2] + head * ost[3];
  const int S = args.split;
  for (int idx = threadIdx.x; idx < kBlockM * 16; idx += 256) {
    const int r = idx >> 4;
    const int c = (idx & 15) * 8;
    if (r >= valid) continue;
    float mx = -INFINITY;
    for (int p = 0; p < S; ++p) mx = fmaxf(mx, args.ws_lse[((u * S + p) * 2 + t) * kBlockM + r]);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float wsum = 0.f;
    for (int p = 0; p < S; ++p) {
      const float lse = args.ws_lse[((u * S + p) * 2 + t) * kBlockM + r];
      const float w = lse == -INFINITY ? 0.f : ex2_approx(lse - mx);
      wsum += w;
      const float4* src = reinterpret_cast<const float4*>(
          args.ws_o + ((static_cast<int64_t>(u * S + p) * 2 + t) * kBlockM + r) * kHeadDim + c);
      const float4 a0 = src[0], a1 = src[1];
      acc[0] = fmaf(w, a0.x, acc[0]);
      acc[1] = fmaf(w, a0.y, acc[1]);
      acc[2] = fmaf(w, a0.z, acc[2]);
      acc[3] = fmaf(w, a0.w, acc[3]);
      acc[4] = fmaf(w, a1.x, acc[4]);
      acc[5] = fmaf(w, a1.y, acc[5]);
      acc[6] = fmaf(w, a1.z, acc[6]);
      acc[7] = fmaf(w, a1.w, acc[7]);
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    const int64_t oidx = otile + static_cast<int64_t>(r) * ost[2] + c;
    if (args.out_fp32) {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(obase) + oidx);
      dst[0] = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
      dst[1] = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
    } else {
      uint4 v;
      v.x = pack2<kFp16>(acc[0] * inv, acc[1] * inv);
      v.y = pack2<kFp16>(acc[2] * inv, acc[3] * inv);
      v.z = pack2<kFp16>(acc[4] * inv, acc[5] * inv);
      v.w = pack2<kFp16>(acc[6] * inv, acc[7] * inv);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(obase) + oidx) = v;
    }
  }
}

}  // namespace attn

namespace {
// Raises the kernel's dynamic shared memory limit once per device (outside
// any stream capture that may follow: the first launch on a device does it).
template <bool kFp16>
int prepare_kernel() {
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (done[dev]) return 0;
  const cudaError_t err = cudaFuncSetAttribute(attn::attn_fwd_kernel<kFp16>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, attn::kSmemBytes);
  if (err != cudaSuccess) return set_cuda_error("attention: cudaFuncSetAttribute", err);
  done[dev] = true;
  return 0;
}
}  // namespace

int launch_attention(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                     const CUtensorMap& tqp, const CUtensorMap& tkp, const CUtensorMap& tvp,
                     const AttnArgs& args, int64_t total_units, bool fp16, cudaStream_t stream) {
  using namespace attn;
  const int64_t split_units = args.split > 1 ? total_units - args.full_units : 0;
  const int64_t ctas = split_units > 0 ? args.full_units + split_units * args.split : total_units;
  if (ctas <= 0) return 0;
  if (ctas > 0x7fffffff) return set_error(PS_B200_ERR_UNSUPPORTED, "attention grid above 2^31 CTAs");
  const dim3 grid(static_cast<unsigned>(ctas));
  const dim3 block(kThreads);
  if (fp16) {
    if (int rc = prepare_kernel<true>()) return rc;
    attn_fwd_kernel<true><<<grid, block, kSmemBytes, stream>>>(tq, tk, tv, tqp, tkp, tvp, args);
  } else {
    if (int rc = prepare_kernel<false>()) return rc;
    attn_fwd_kernel<false><<<grid, block, kSmemBytes, stream>>>(tq, tk, tv, tqp, tkp, tvp, args);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_cuda_error("attention launch", err);
  count_launch();
  if (split_units > 0) {
    const dim3 cgrid(static_cast<unsigned>(split_units * 2));
    if (fp16)
      attn_combine_kernel<true><<<cgrid, 256, 0, stream>>>(args);
    else
      attn_combine_kernel<false><<<cgrid, 256, 0, stream>>>(args);
    err = cudaGetLastError();
    if (err != cudaSuccess) return set_cuda_error("attention combine launch", err);
    count_launch();
  }
  return 0;
}

}  // namespace psb
