// K2: attention backward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces `attention_backward` (kotflash/kernels/triton_backward.py:335-421)
// and its kernels `_attention_bwd_dq` (:18-91), `_attention_bwd_dkv` (:95-195),
// `_attention_bwd_dkv_split` (:199-312) and `_attention_bwd_dkv_reduce`
// (:315-332).  Same math as the reference's blockwise backward
// (kotflash/attention.py:138-201): P = exp(scale*QK^T - LSE),
// dP = dO V^T, Delta = rowsum(O*dO), dS = P (dP - Delta), dQ = scale dS K,
// dK = scale dS^T Q, dV = P^T dO, dK/dV summed over the GQA group.
//
// Three launches:
//   1. prep   : Delta and LSE*log2(e) per query row (rows padded to 64; padded
//               rows get LSE = +inf so their P is exactly 0); dQ workspace zeroed.
//   2. main   : one CTA per (batch, KV head, 128-key block).  K and V stay in
//               shared memory; the CTA walks every query head of the group and
//               every 64-row query block that can see its keys.  Per step:
//                 S^T  = K Q^T      (SS MMA, M=128 keys, N=64 rows)
//                 dP^T = V dO^T     (SS MMA)
//                 softmax warps (thread = key), in two phases: P^T as soon as
//                 S^T is ready, dS^T = P^T (dP^T - Delta) once dP^T is, each
//                 written to TMEM as 16-bit; dS^T also to shared memory
//                 (128-byte swizzled, q contiguous)
//                 dV  += P^T dO     (TS MMA, A = P^T in TMEM)
//                 dK  += dS^T Q     (TS MMA, A = dS^T in TMEM)
//                 dQ^T = K^T dS^T   (SS MMA, both operands MN-major)
//               Two threads issue the MMAs: one the score GEMMs (S^T, dP^T),
//               one the gradient GEMMs (dV, dK, dQ^T).  On sm_100 the tensor
//               pipe keeps almost no MMAs queued, so the barrier waits, fences
//               and commits of a single issuing thread would idle it; with two
//               issuers each one's synchronisation is covered by the other's
//               MMAs.  S^T/P^T and dP^T/dS^T are double-buffered in TMEM and
//               dS^T in shared memory; dQ^T(s) is written over the dP^T/dS^T
//               buffer of its own step once dK(s) has read it (MMAs of one
//               thread execute in order), which is what frees the TMEM for
//               the second S^T buffer.  Every loop-carried dependency thus
//               spans two steps.
//               dQ^T (thread = head-dim lane) is
//               staged in 128-byte swizzled shared memory by a dedicated
//               warpgroup and added into the fp32 workspace with TMA
//               reduce-add (cp.reduce.async.bulk.tensor), off the LSU path.  dK/dV accumulate in TMEM for the whole group and are
//               written once, so no dK/dV partial buffers exist.
//   3. finish : dQ = scale * workspace, cast to the input dtype.
// Tensor memory (512 columns): dV [0,128) dK [128,256), S^T/P^T buffers
// [256,320) [320,384), dP^T/dS^T/dQ^T buffers [384,448) [448,512).
// Warps: 0-7 softmax (two warpgroups split the 64 query columns), 8-11 dQ
// drain, 12 TMA producer, 13 TMEM allocator + score-GEMM issuer, 14
// gradient-GEMM issuer; 0-7 also write the dV (warps 0-3) and dK (warps 4-7)
// epilogue.
#include <math.h>

#include <algorithm>

#include "kf_host.h"
#include "kf_sm100.cuh"

namespace {

constexpr int kBM = 64;    // query rows per step
constexpr int kBN = 128;   // keys per CTA
constexpr int kStages = 3;  // Q/dO/statistics ring
constexpr int kThreads = 480;  // 15 warps
// (batch, KV head) pairs per launch group of the main kernel: with 8 the
// greedy block scheduler ends the grid as evenly as the global
// heaviest-first order does (a simulation of the causal 4096-token config
// over 148 SMs: 928 step-times either way, 968 with 4 pairs, 1056 with 1).
#ifndef KF_BWD_PAIRS_PER_GROUP
#define KF_BWD_PAIRS_PER_GROUP 8
#endif
constexpr int kPairsPerGroup = KF_BWD_PAIRS_PER_GROUP;
// TMEM columns
constexpr uint32_t kColDV = 0, kColDK = 128, kColS = 256, kColDP = 384;
// 16-bit P^T / dS^T of query columns [32 wg, 32 wg + 32) are packed into the
// first 16 of the 32 fp32 columns that held that warpgroup's S^T / dP^T, so a
// warpgroup never overwrites columns the other one still has to read.  MMA
// k-step kk (16 queries) therefore reads packed column 32 (kk / 2) + 8 (kk % 2).
__host__ __device__ constexpr uint32_t packed_col(int kk) { return 32u * (kk >> 1) + 8u * (kk & 1); }
constexpr float kLog2e = 1.4426950408889634f;
#ifndef KF_BWD_POLY_QUADS
#define KF_BWD_POLY_QUADS 0
#endif
constexpr int kPolyQuads = KF_BWD_POLY_QUADS;

struct BwdParams {
  uint16_t* dk;
  uint16_t* dv;
  int64_t dks[4], dvs[4];
  float* dq_acc;          // [B*Hq][nqb][D][64]
  const float* lse2;      // [B*Hq][Sq_pad] LSE * log2(e); +inf on padded rows
  const float* delta;     // [B*Hq][Sq_pad]
  int B, Hq, Hkv, G, Sq, Sk, D, Sq_pad, nqb, nkb;
  int pairs_per_group;    // (batch, KV head) pairs whose CTAs are launched together
  // Query split of a key block over several CTAs (1 = none): key block n's
  // query blocks are cut into ceil(blocks / part_chunk) near-equal parts,
  // one CTA each (CTAs whose part does not exist return at once), and every
  // part adds its fp32 dK/dV into dkv_acc ([B*Hkv*Sk_pad][D] for dK, then
  // the same for dV) with TMA reduce-add.
  int parts_max, part_chunk, Sk_pad;
  int causal;
  float scale_log2, scale;
  int32_t* status;
};

struct __align__(8) BwdBarriers {
  uint64_t kv_full;
  uint64_t qdo_full[kStages], qdo_empty[kStages];
  uint64_t s_ready[2], p_ready[2], p_free[2];     // per S^T/P^T buffer
  uint64_t dp_ready[2], ds_ready[2], dq_full[2];  // per dP^T/dS^T/dQ^T buffer
  uint64_t ds_free[2];                            // dQ^T drained: buffer reusable
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, BwdBarriers* bars,
                                         int32_t* status) {
  if (kf::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = kf::global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (kf::mbar_try_wait_sleep(bar, parity, 20000)) return true;
    if ((++spins & 15u) == 0) {
      if (*(volatile int*)&bars->abort_flag) return false;
      if (kf::global_timer_ns() - t0 > kf::kWaitBudgetNs) {
        *(volatile int*)&bars->abort_flag = 1;
        if (status) atomicExch(status, KF_DEV_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          kf::smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(kf::smem_u32(bar))
      : "memory");
}

template <bool BF16, int KS>
__global__ void __launch_bounds__(kThreads, 1)
bwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
           const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_do,
           const __grid_constant__ CUtensorMap map_dq, const __grid_constant__ CUtensorMap map_dk,
           const __grid_constant__ CUtensorMap map_dv, const BwdParams p) {
  constexpr int KPANEL = kBN * 128;  // 16 KB: 128 rows x 64 columns
  constexpr int QPANEL = kBM * 128;  // 8 KB: 64 rows x 64 columns
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sK = smem;                               // 2 panels
  uint8_t* sV = sK + 2 * KPANEL;                    // 2 panels
  uint8_t* sQ = sV + 2 * KPANEL;                    // [stage][2 panels]
  uint8_t* sdO = sQ + kStages * 2 * QPANEL;         // [stage][2 panels]
  uint8_t* sdS = sdO + kStages * 2 * QPANEL;        // [2 buffers][128 rows x 128 B]
  uint8_t* sDQ = sdS + 2 * KPANEL;                  // [2 halves][D rows][32 fp32]
  float* sLD = reinterpret_cast<float*>(sDQ + 2 * 128 * 128);  // [stage][lse2 64 | delta 64]
  BwdBarriers* bars = reinterpret_cast<BwdBarriers*>(sLD + kStages * 2 * kBM);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // CTA order: the (batch, KV head) pairs go in groups of pairs_per_group;
  // inside a group every CTA of key block 0 (the most causal work) launches
  // before any of key block 1, and so on, so each group (and the grid) ends
  // on light CTAs.  Every CTA walks its query blocks from the last one down,
  // one block at a time over the group's heads, so the CTAs of one pair,
  // launched together, add into the same dQ accumulator tiles and read the
  // same Q/dO tiles at about the same time: each tile passes through DRAM
  // about once instead of once per wave of key blocks.
  const int n_pairs = p.B * p.Hkv;
  const int per_group = p.pairs_per_group * p.nkb * p.parts_max;
  const int grp = (int)blockIdx.x / per_group;
  int rem = (int)blockIdx.x - grp * per_group;
  const int part = rem % p.parts_max;
  rem /= p.parts_max;
  const int gp = min(p.pairs_per_group, n_pairs - grp * p.pairs_per_group);
  const int n = rem / gp;
  const int bkv = grp * p.pairs_per_group + rem % gp;
  const int b = bkv / p.Hkv, kvh = bkv % p.Hkv;
  const int i0 = p.causal ? min((n * kBN) / kBM, p.nqb) : 0;
  const int nq_all = p.nqb - i0;  // query blocks that see this key block
  const bool split = p.parts_max > 1;
  const int nparts = split ? (nq_all + p.part_chunk - 1) / p.part_chunk : 1;
  if (split && part >= nparts) return;  // no such part: nothing to do (dK/dV accumulators start at zero)
  // this CTA's query blocks, in sweep order: [u0, u1) of the nq_all blocks
  const int u0 = (int)((int64_t)part * nq_all / nparts);
  const int u1 = (int)((int64_t)(part + 1) * nq_all / nparts);
  const int s_begin = p.G * u0;         // first (global) step of this CTA
  const int nsteps = p.G * (u1 - u0);   // loops below count local steps 0 .. nsteps - 1
  constexpr int d_pad16 = KS * 16;  // head dim rounded up to the MMA K step

  if (tid == 0) {
    kf::mbar_init(&bars->kv_full, 1);
    for (int s = 0; s < kStages; ++s) {
      kf::mbar_init(&bars->qdo_full[s], 1);
      kf::mbar_init(&bars->qdo_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      kf::mbar_init(&bars->s_ready[s], 1);
      kf::mbar_init(&bars->p_ready[s], 256);
      kf::mbar_init(&bars->p_free[s], 1);
      kf::mbar_init(&bars->dp_ready[s], 1);
      kf::mbar_init(&bars->ds_ready[s], 256);
      kf::mbar_init(&bars->dq_full[s], 1);
      kf::mbar_init(&bars->ds_free[s], 128);
    }
    kf::mbar_init(&bars->mma_done, 1);
    bars->abort_flag = 0;
    kf::fence_barrier_init();
  }
  if (warp == 13) {
    kf::tmem_alloc(&bars->tmem_base, 512);
    kf::tmem_relinquish();
  }
  kf::tc_fence_before();
  __syncthreads();
  kf::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // local step s = global step s_begin + s: query block nqb - 1 - (global step) / G
  // (last block first), head (global step) % G of the group
  auto step_coords = [&](int s, int& h, int& i) {
    const int gs = s_begin + s;
    h = kvh * p.G + gs % p.G;
    i = p.nqb - 1 - gs / p.G;
  };

  if (warp == 12) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && nsteps > 0) {
      kf::mbar_arrive_expect_tx(&bars->kv_full, 4 * KPANEL);
      for (int pn = 0; pn < 2; ++pn) {
        kf::tma_load_4d(sK + pn * KPANEL, &map_k, &bars->kv_full, pn * 64, n * kBN, kvh, b);
        kf::tma_load_4d(sV + pn * KPANEL, &map_v, &bars->kv_full, pn * 64, n * kBN, kvh, b);
      }
      for (int s = 0; s < nsteps; ++s) {
        const int st = s % kStages;
        if (!wait_bar(&bars->qdo_empty[st], ((s / kStages) & 1) ^ 1, bars, p.status)) break;
        int h, i;
        step_coords(s, h, i);
        kf::mbar_arrive_expect_tx(&bars->qdo_full[st], 4 * QPANEL + 2 * kBM * 4);
        for (int pn = 0; pn < 2; ++pn) {
          kf::tma_load_4d(sQ + (st * 2 + pn) * QPANEL, &map_q, &bars->qdo_full[st], pn * 64, i * kBM, h, b);
          kf::tma_load_4d(sdO + (st * 2 + pn) * QPANEL, &map_do, &bars->qdo_full[st], pn * 64, i * kBM, h, b);
        }
        const int64_t row_off = ((int64_t)b * p.Hq + h) * p.Sq_pad + (int64_t)i * kBM;
        bulk_load(sLD + st * 2 * kBM, p.lse2 + row_off, kBM * 4, &bars->qdo_full[st]);
        bulk_load(sLD + st * 2 * kBM + kBM, p.delta + row_off, kBM * 4, &bars->qdo_full[st]);
      }
    }
  } else if (warp == 13 || warp == 14) {
    // ------------------------------------------------------------ MMA issuers
    if (lane == 0 && nsteps > 0) {
      const uint32_t idesc_s = kf::make_idesc_f16(BF16, 128, kBM, 0, 0);
      const uint32_t idesc_kv = kf::make_idesc_f16(BF16, 128, d_pad16, 0, 1);
      const uint32_t idesc_q = kf::make_idesc_f16(BF16, 128, kBM, 1, 1);
      // Descriptors are built once; each MMA adds a compile-time offset.
      const kf::SDesc dk_k = kf::make_sdesc_split(kf::smem_u32(sK), 16, 1024);
      const kf::SDesc dk_v = kf::make_sdesc_split(kf::smem_u32(sV), 16, 1024);
      const kf::SDesc dk_q = kf::make_sdesc_split(kf::smem_u32(sQ), 16, 1024);
      const kf::SDesc dk_do = kf::make_sdesc_split(kf::smem_u32(sdO), 16, 1024);
      const kf::SDesc dm_q = kf::make_sdesc_split(kf::smem_u32(sQ), QPANEL, 1024);
      const kf::SDesc dm_do = kf::make_sdesc_split(kf::smem_u32(sdO), QPANEL, 1024);
      const kf::SDesc dm_k = kf::make_sdesc_split(kf::smem_u32(sK), KPANEL, 1024);
      const kf::SDesc dm_ds = kf::make_sdesc_split(kf::smem_u32(sdS), KPANEL, 1024);
      bool ok = wait_bar(&bars->kv_full, 0, bars, p.status);
      if (warp == 13) {
        // score GEMMs: S^T(s) = K Q^T, dP^T(s) = V dO^T into buffer s & 1
        for (int s = 0; ok && s < nsteps; ++s) {
          const int st = s % kStages, buf = s & 1;
          const uint32_t qoff = st * 2 * QPANEL;
          if (!(ok = wait_bar(&bars->qdo_full[st], (s / kStages) & 1, bars, p.status))) break;
          // P^T(s-2), which overlays S^T in this buffer, has been read by dV(s-2)
          if (s >= 2 && !(ok = wait_bar(&bars->p_free[buf], ((s - 2) >> 1) & 1, bars, p.status))) break;
          kf::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < KS; ++kk) {
            const uint32_t ka = (kk >> 2) * KPANEL + (kk & 3) * 32;
            const uint32_t qa = (kk >> 2) * QPANEL + (kk & 3) * 32;
            kf::umma_ss(tmem + kColS + buf * 64, kf::sdesc_at(dk_k, ka), kf::sdesc_at(dk_q, qoff + qa),
                        idesc_s, kk > 0);
          }
          kf::umma_commit(&bars->s_ready[buf]);
          // dQ^T(s-2) has been drained from buffer `buf` (so dK(s-2) and
          // dQ^T(s-2) are also done with dS^T(s-2) in TMEM and shared memory)
          if (s >= 2 && !(ok = wait_bar(&bars->ds_free[buf], ((s - 2) >> 1) & 1, bars, p.status))) break;
          kf::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < KS; ++kk) {
            const uint32_t ka = (kk >> 2) * KPANEL + (kk & 3) * 32;
            const uint32_t qa = (kk >> 2) * QPANEL + (kk & 3) * 32;
            kf::umma_ss(tmem + kColDP + buf * 64, kf::sdesc_at(dk_v, ka), kf::sdesc_at(dk_do, qoff + qa),
                        idesc_s, kk > 0);
          }
          kf::umma_commit(&bars->dp_ready[buf]);
        }
      } else {
        // gradient GEMMs: dV += P^T dO, dK += dS^T Q, dQ^T = K^T dS^T
        for (int s = 0; ok && s < nsteps; ++s) {
          const int st = s % kStages, buf = s & 1;
          const uint32_t qoff = st * 2 * QPANEL;
          if (!(ok = wait_bar(&bars->p_ready[buf], (s >> 1) & 1, bars, p.status))) break;
          kf::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            kf::umma_ts(tmem + kColDV, tmem + kColS + buf * 64 + packed_col(kk),
                        kf::sdesc_at(dm_do, qoff + kk * 2048), idesc_kv, (s > 0 || kk > 0));
          kf::umma_commit(&bars->p_free[buf]);
          if (!(ok = wait_bar(&bars->ds_ready[buf], (s >> 1) & 1, bars, p.status))) break;
          kf::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            kf::umma_ts(tmem + kColDK, tmem + kColDP + buf * 64 + packed_col(kk),
                        kf::sdesc_at(dm_q, qoff + kk * 2048), idesc_kv, (s > 0 || kk > 0));
          kf::umma_commit(&bars->qdo_empty[st]);
          // dQ^T(s) overwrites this step's dS^T in TMEM after dK(s) read it
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk)
            kf::umma_ss(tmem + kColDP + buf * 64, kf::sdesc_at(dm_k, kk * 2048),
                        kf::sdesc_at(dm_ds, buf * KPANEL + kk * 2048), idesc_q, kk > 0);
          kf::umma_commit(&bars->dq_full[buf]);
        }
        kf::umma_commit(&bars->mma_done);
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ P / dS (thread = key)
    // two warpgroups: wg 0 takes query columns [0, 32), wg 1 takes [32, 64)
    const int wg = warp >> 2;
    const int c0 = wg * 32;
    const int kr = (warp & 3) * 32 + lane;
    const int key = n * kBN + kr;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    bool ok = true;
    for (int s = 0; ok && s < nsteps; ++s) {
      const int i_step = p.nqb - 1 - (s_begin + s) / p.G;  // query block of step s (see step_coords)
      const int st = s % kStages, buf = s & 1;
      if (!(ok = wait_bar(&bars->qdo_full[st], (s / kStages) & 1, bars, p.status))) break;
      // The row statistics are read into registers before waiting for S^T:
      // during the step the tensor cores keep shared memory busy, and a load
      // issued after S^T is ready would sit on the critical path.
      const float4* lse4 = reinterpret_cast<const float4*>(sLD + st * 2 * kBM + c0);
      const float4* dlt4 = reinterpret_cast<const float4*>(sLD + st * 2 * kBM + kBM + c0);
      float4 lv[8];
#pragma unroll
      for (int c4 = 0; c4 < 8; ++c4) lv[c4] = lse4[c4];
      const int q0 = i_step * kBM + c0;
      const uint32_t col_s = kColS + buf * 64;
      if (!(ok = __all_sync(0xffffffffu, wait_bar(&bars->s_ready[buf], (s >> 1) & 1, bars, p.status)))) break;
      kf::tc_fence_after();
      uint32_t sr[32];
      kf::tmem_ld32(lane_base + col_s + c0, sr);
      kf::tmem_wait_ld();
      // visible iff key < Sk and (not causal or key <= q): columns c >= first_q
      const int first_q = p.causal ? key - q0 : 0;
      const bool key_ok = key < p.Sk;
      float pr[32];
      // kPolyQuads of the 8 groups of four exponentials run as the fp32-pipe
      // polynomial, the rest on MUFU (x <= 0 here; padded rows give x = -inf,
      // which the polynomial clamps to a ~2^-125 P that meets zero dO / dP).
#pragma unroll
      for (int c4 = 0; c4 < 8; ++c4) {
        const float4 l = lv[c4];
        const float x0 = __uint_as_float(sr[4 * c4 + 0]) * p.scale_log2 - l.x;
        const float x1 = __uint_as_float(sr[4 * c4 + 1]) * p.scale_log2 - l.y;
        const float x2 = __uint_as_float(sr[4 * c4 + 2]) * p.scale_log2 - l.z;
        const float x3 = __uint_as_float(sr[4 * c4 + 3]) * p.scale_log2 - l.w;
        if (c4 < kPolyQuads) {
          kf::f2_split(kf::exp2_poly2(x0, x1), pr[4 * c4 + 0], pr[4 * c4 + 1]);
          kf::f2_split(kf::exp2_poly2(x2, x3), pr[4 * c4 + 2], pr[4 * c4 + 3]);
        } else {
          pr[4 * c4 + 0] = kf::ex2(x0);
          pr[4 * c4 + 1] = kf::ex2(x1);
          pr[4 * c4 + 2] = kf::ex2(x2);
          pr[4 * c4 + 3] = kf::ex2(x3);
        }
      }
      if (!key_ok || first_q > 0) {  // only blocks on the causal diagonal or past Sk
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (!key_ok || c < first_q) pr[c] = 0.f;
      }
      uint32_t pk[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) pk[c] = kf::pack2<BF16>(pr[2 * c], pr[2 * c + 1]);
      kf::tmem_st16(lane_base + col_s + c0, pk);  // over this warpgroup's own S^T columns
      kf::tmem_wait_st();
      kf::tc_fence_before();
      kf::mbar_arrive(&bars->p_ready[buf]);

      const uint32_t col_dp = kColDP + buf * 64;
#pragma unroll
      for (int c4 = 0; c4 < 8; ++c4) lv[c4] = dlt4[c4];
      if (!(ok = __all_sync(0xffffffffu, wait_bar(&bars->dp_ready[buf], (s >> 1) & 1, bars, p.status)))) break;
      kf::tc_fence_after();
      uint32_t dr[32];
      kf::tmem_ld32(lane_base + col_dp + c0, dr);
      kf::tmem_wait_ld();
      uint32_t dk[16];
#pragma unroll
      for (int c4 = 0; c4 < 8; ++c4) {
        const float4 dl = lv[c4];
        dk[2 * c4] = kf::pack2<BF16>(pr[4 * c4 + 0] * (__uint_as_float(dr[4 * c4 + 0]) - dl.x),
                                     pr[4 * c4 + 1] * (__uint_as_float(dr[4 * c4 + 1]) - dl.y));
        dk[2 * c4 + 1] = kf::pack2<BF16>(pr[4 * c4 + 2] * (__uint_as_float(dr[4 * c4 + 2]) - dl.z),
                                         pr[4 * c4 + 3] * (__uint_as_float(dr[4 * c4 + 3]) - dl.w));
      }
      kf::tmem_st16(lane_base + col_dp + c0, dk);  // over this warpgroup's own dP^T columns
      // dS^T row -> shared memory, 128-byte swizzle (16-byte chunk c at c ^ (row & 7))
      uint8_t* row_ptr = sdS + buf * KPANEL + kr * 128;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(row_ptr + (((wg * 4 + j) ^ (kr & 7)) << 4)) =
            make_uint4(dk[4 * j], dk[4 * j + 1], dk[4 * j + 2], dk[4 * j + 3]);
      kf::fence_proxy_async_smem();
      kf::tmem_wait_st();
      kf::tc_fence_before();
      kf::mbar_arrive(&bars->ds_ready[buf]);
    }
  } else if (warp < 12) {
    // ------------------------------------------------------------ dQ drain (thread = head-dim lane)
    // TMEM -> swizzled shared staging tile -> TMA reduce-add into the fp32 workspace
    const int dl = (warp - 8) * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)((warp - 8) * 32) << 16);
    const int d_rows = p.D;                 // multiple of 8, so halves stay 1024-aligned
    bool ok = true;
    for (int s = 0; ok && s < nsteps; ++s) {
      const int buf = s & 1;  // TMEM buffer and shared-memory staging buffer
      // one decision for the whole warpgroup (its named barriers below must
      // see every thread), even if one thread's bounded wait gave up
      ok = kf::named_bar_and(1, 128, wait_bar(&bars->dq_full[buf], (s >> 1) & 1, bars, p.status));
      if (!ok) break;
      kf::tc_fence_after();
      uint32_t v[64];
      kf::tmem_ld32(lane_base + kColDP + buf * 64, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      kf::tmem_ld32(lane_base + kColDP + buf * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      kf::tmem_wait_ld();
      kf::tc_fence_before();
      kf::mbar_arrive(&bars->ds_free[buf]);
      // The staging tile has two halves (query columns 0-31 and 32-63), each
      // reduced by its own bulk group, so the reduce of one half overlaps
      // the staging of the other.
      int row0 = 0;
      if (dl == 0) {
        int h, i;
        step_coords(s, h, i);
        row0 = (int)((((int64_t)b * p.Hq + h) * p.nqb + i) * p.D);
      }
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint8_t* half = sDQ + hf * d_rows * 128;
        // this half was last reduced two bulk groups ago
        if (dl == 0) kf::bulk_wait_group_read<1>();
        kf::named_bar_sync(1, 128);
        if (dl < d_rows) {
          uint8_t* row_ptr = half + dl * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(row_ptr + ((c ^ (dl & 7)) << 4)) =
                make_uint4(v[hf * 32 + 4 * c], v[hf * 32 + 4 * c + 1], v[hf * 32 + 4 * c + 2],
                           v[hf * 32 + 4 * c + 3]);
        }
        kf::fence_proxy_async_smem();
        kf::named_bar_sync(1, 128);
        if (dl == 0) {
          kf::tma_reduce_add_2d(&map_dq, half, hf * 32, row0);
          kf::bulk_commit_group();
        }
      }
    }
    if (dl == 0) kf::bulk_wait_group<0>();
  }

  // ---------------------------------------------------------- dK / dV epilogue
  if (warp < 8) {
    const bool is_dk = warp >= 4;
    const int kr = (warp & 3) * 32 + lane;
    const int key = n * kBN + kr;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    uint16_t* dst = is_dk ? p.dk + b * p.dks[0] + (int64_t)kvh * p.dks[1] + (int64_t)key * p.dks[2]
                          : p.dv + b * p.dvs[0] + (int64_t)kvh * p.dvs[1] + (int64_t)key * p.dvs[2];
    const float mul = is_dk ? p.scale : 1.f;
    const bool have = __all_sync(0xffffffffu, nsteps > 0 && wait_bar(&bars->mma_done, 0, bars, p.status));
    if (have) kf::tc_fence_after();
    if (split) {
      // This CTA's part of dK/dV goes to the fp32 accumulators: each
      // warpgroup stages its tensor as 128-row x 32-column fp32 boxes
      // (128-byte swizzle) in shared memory no MMA or TMA load uses any more
      // (dV over the Q/dO ring, dK over K/V) and one thread adds the boxes
      // with TMA reduce-add; the finish kernel converts the sums.
      uint8_t* stage = is_dk ? sK : sQ;
      if (have) {
#pragma unroll
        for (int c0 = 0; c0 < d_pad16; c0 += 64) {
          uint32_t ov[64];
          const bool two = c0 + 32 < d_pad16;
          kf::tmem_ld32(lane_base + (is_dk ? kColDK : kColDV) + c0, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
          if (two)
            kf::tmem_ld32(lane_base + (is_dk ? kColDK : kColDV) + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[32]));
          kf::tmem_wait_ld();
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            if (hb == 1 && !two) break;
            uint8_t* row_ptr = stage + ((c0 >> 5) + hb) * (kBN * 128) + kr * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<uint4*>(row_ptr + ((j ^ (kr & 7)) << 4)) =
                  make_uint4(ov[32 * hb + 4 * j], ov[32 * hb + 4 * j + 1], ov[32 * hb + 4 * j + 2],
                             ov[32 * hb + 4 * j + 3]);
          }
        }
        kf::fence_proxy_async_smem();
      }
      kf::named_bar_sync(is_dk ? 3 : 2, 128);
      if (have && (warp & 3) == 0 && lane == 0) {
        const int row0 = bkv * p.Sk_pad + n * kBN;
        for (int c0 = 0; c0 < d_pad16; c0 += 32)
          kf::tma_reduce_add_2d(is_dk ? &map_dk : &map_dv, stage + (c0 >> 5) * (kBN * 128), c0, row0);
        kf::bulk_commit_group();
        kf::bulk_wait_group<0>();
      }
    } else if (nsteps == 0 || have) {
      // 64-column batches: two TMEM loads in flight per wait
#pragma unroll
      for (int c0 = 0; c0 < d_pad16; c0 += 64) {
        uint32_t ov[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) ov[c] = 0u;
        if (have) {
          kf::tmem_ld32(lane_base + (is_dk ? kColDK : kColDV) + c0, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
          if (c0 + 32 < d_pad16)
            kf::tmem_ld32(lane_base + (is_dk ? kColDK : kColDV) + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[32]));
          kf::tmem_wait_ld();
        }
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c)
          pk[c] = kf::pack2<BF16>(__uint_as_float(ov[2 * c]) * mul, __uint_as_float(ov[2 * c + 1]) * mul);
        if (key < p.Sk) {
#pragma unroll
          for (int g8 = 0; g8 < 8; ++g8)
            if (c0 + g8 * 8 < p.D)
              *reinterpret_cast<uint4*>(dst + c0 + g8 * 8) =
                  make_uint4(pk[4 * g8], pk[4 * g8 + 1], pk[4 * g8 + 2], pk[4 * g8 + 3]);
        }
      }
    }
  }

  kf::tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    kf::tc_fence_after();
    kf::tmem_dealloc(tmem, 512);
  }
}

// Delta = rowsum(O * dO) and LSE * log2(e) per (padded) query row, plus the
// zero fill of the fp32 dQ accumulator.  Sixteen threads share a row (16-byte
// loads of O and dO, eight elements each); the grid strides over rows so
// every SM keeps many loads in flight.
struct PrepArgs {
  const uint16_t* o;
  const uint16_t* dout;
  const float* lse;
  float* lse2;
  float* delta;
  float4* acc;         // dQ accumulator, zeroed here
  int64_t acc_vec4;    // its length in float4
  float4* acc2;        // dK/dV accumulators when key blocks are split (else null), zeroed here
  int64_t acc2_vec4;
  int64_t os[4], dos[4];
  int Hq, Sq, Sq_pad, D;
  int64_t rows;  // B*Hq*Sq_pad
};

template <bool BF16>
__global__ void __launch_bounds__(256) prep_kernel(const PrepArgs a) {
  const int sub = threadIdx.x & 15;
  const int64_t stride = (int64_t)gridDim.x * 16;
  for (int64_t row = (int64_t)blockIdx.x * 16 + (threadIdx.x >> 4); row - (threadIdx.x >> 4) < a.rows;
       row += stride) {
    // every thread of a warp reaches the shuffles below, rows past the end included
    const bool in = row < a.rows;
    const int64_t bh = in ? row / a.Sq_pad : 0;
    const int q = in ? (int)(row % a.Sq_pad) : 0;
    const bool real = in && q < a.Sq;
    float acc = 0.f;
    if (real && sub * 8 < a.D) {
      const int64_t b = bh / a.Hq, h = bh % a.Hq;
      const uint4 ov = *reinterpret_cast<const uint4*>(a.o + b * a.os[0] + h * a.os[1] + (int64_t)q * a.os[2] + sub * 8);
      const uint4 dv = *reinterpret_cast<const uint4*>(a.dout + b * a.dos[0] + h * a.dos[1] + (int64_t)q * a.dos[2] + sub * 8);
      const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 o2 = kf::unpack2<BF16>(ow[j]), d2 = kf::unpack2<BF16>(dw[j]);
        acc += o2.x * d2.x + o2.y * d2.y;
      }
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (in && sub == 0) {
      a.delta[row] = real ? acc : 0.f;
      a.lse2[row] = real ? a.lse[bh * a.Sq + q] * kLog2e : INFINITY;
    }
  }
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < a.acc_vec4; i += (int64_t)gridDim.x * 256)
    a.acc[i] = z;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < a.acc2_vec4; i += (int64_t)gridDim.x * 256)
    a.acc2[i] = z;
}

// dQ = scale * workspace ([bh][qb][D][64] fp32) -> dq [B,Hq,Sq,D] in the input
// dtype: one block per 64-row tile, transposed through shared memory, written
// with 16-byte row-contiguous stores.
struct FinishArgs {
  const float* acc;
  uint16_t* dq;
  int64_t qs[4];
  int Hq, Sq, D, nqb;
  float scale;
};

template <bool BF16>
__global__ void __launch_bounds__(256) finish_kernel(const FinishArgs a) {
  __shared__ float tile[kBM][128 + 1];  // [query][d]
  const int qb = blockIdx.x, bh = blockIdx.y;
  const float4* src = reinterpret_cast<const float4*>(a.acc + ((int64_t)bh * a.nqb + qb) * a.D * kBM);
  for (int idx = threadIdx.x; idx < a.D * (kBM / 4); idx += 256) {
    const int d = idx / (kBM / 4), q4 = (idx % (kBM / 4)) * 4;
    const float4 v = src[idx];
    tile[q4 + 0][d] = v.x;
    tile[q4 + 1][d] = v.y;
    tile[q4 + 2][d] = v.z;
    tile[q4 + 3][d] = v.w;
  }
  __syncthreads();
  const int b = bh / a.Hq, h = bh % a.Hq;
  const int nd8 = a.D / 8;
  for (int idx = threadIdx.x; idx < kBM * nd8; idx += 256) {
    const int r = idx / nd8, d8 = (idx % nd8) * 8;
    const int q = qb * kBM + r;
    if (q >= a.Sq) continue;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = kf::pack2<BF16>(tile[r][d8 + 2 * j] * a.scale, tile[r][d8 + 2 * j + 1] * a.scale);
    *reinterpret_cast<uint4*>(a.dq + b * a.qs[0] + (int64_t)h * a.qs[1] + (int64_t)q * a.qs[2] + d8) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// dK = scale * acc_k, dV = acc_v ([B*Hkv*Sk_pad][D] fp32 sums of the split
// parts) -> the caller's dk/dv in the input dtype: eight consecutive columns
// of one key row per thread, 16-byte stores.
struct FinishKVArgs {
  const float* acc_k;
  const float* acc_v;
  uint16_t* dk;
  uint16_t* dv;
  int64_t dks[4], dvs[4];
  int Hkv, Sk, Sk_pad, D;
  float scale;
  int64_t rows;  // B*Hkv*Sk
};

template <bool BF16>
__global__ void __launch_bounds__(256) finish_kv_kernel(const FinishKVArgs a) {
  const int nd8 = a.D / 8;
  for (int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x; idx < 2 * a.rows * nd8;
       idx += (int64_t)gridDim.x * 256) {
    const bool is_v = idx >= a.rows * nd8;
    const int64_t li = is_v ? idx - a.rows * nd8 : idx;
    const int64_t row = li / nd8;
    const int d8 = (int)(li % nd8) * 8;
    const int64_t bh = row / a.Sk;
    const int key = (int)(row % a.Sk);
    const float* src = (is_v ? a.acc_v : a.acc_k) + (bh * a.Sk_pad + key) * a.D + d8;
    const float4 x = reinterpret_cast<const float4*>(src)[0], y = reinterpret_cast<const float4*>(src)[1];
    const float m = is_v ? 1.f : a.scale;
    const int64_t b = bh / a.Hkv, h = bh % a.Hkv;
    const int64_t* st = is_v ? a.dvs : a.dks;
    uint16_t* dst = (is_v ? a.dv : a.dk) + b * st[0] + h * st[1] + (int64_t)key * st[2] + d8;
    *reinterpret_cast<uint4*>(dst) =
        make_uint4(kf::pack2<BF16>(x.x * m, x.y * m), kf::pack2<BF16>(x.z * m, x.w * m),
                   kf::pack2<BF16>(y.x * m, y.y * m), kf::pack2<BF16>(y.z * m, y.w * m));
  }
}

bool rows16(const kf_tensor4* t) {
  if (!t || !kf::aligned16(t->ptr) || t->stride[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (t->size[i] > 1 && (t->stride[i] % 8) != 0) return false;
  return true;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

template <bool BF16, int KS>
int launch_bwd_main(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                    const CUtensorMap& mdo, const CUtensorMap& mdq, const CUtensorMap& mdk,
                    const CUtensorMap& mdv, const BwdParams& p, cudaStream_t st) {
  const size_t smem = 1024 + 4 * 128 * 128 + kStages * 4 * kBM * 128 + 2 * 128 * 128 +
                      2 * 128 * 128 + kStages * 2 * kBM * 4 + sizeof(BwdBarriers);
  auto kern = bwd_kernel<BF16, KS>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return kf::set_error(KF_ERR_CUDA, "kf_attn_bwd: cannot reserve %zu bytes of shared memory", smem);
  const int64_t grid = (int64_t)p.B * p.Hkv * p.nkb * p.parts_max;
  if (grid > 0x7fffffffLL) return kf::set_error(KF_ERR_UNSUPPORTED, "kf_attn_bwd: grid too large");
  kern<<<(unsigned)grid, kThreads, smem, st>>>(mq, mk, mv, mdo, mdq, mdk, mdv, p);
  return kf::check_launch("kf_attn_bwd main");
}

template <bool BF16>
int dispatch_bwd_main(int ks, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                      const CUtensorMap& mdo, const CUtensorMap& mdq, const CUtensorMap& mdk,
                      const CUtensorMap& mdv, const BwdParams& p, cudaStream_t st) {
  switch (ks) {
    case 1: return launch_bwd_main<BF16, 1>(mq, mk, mv, mdo, mdq, mdk, mdv, p, st);
    case 2: return launch_bwd_main<BF16, 2>(mq, mk, mv, mdo, mdq, mdk, mdv, p, st);
    case 3: return launch_bwd_main<BF16, 3>(mq, mk, mv, mdo, mdq, mdk, mdv, p, st);
    case 4: return launch_bwd_main<BF16, 4>(mq, mk, mv, mdo, mdq, mdk, mdv, p, st);
    case 5: return launch_bwd_main<BF16, 5>(mq, mk, mv, mdo, mdq, mdk, mdv, p, st);
    case 6: return launch_bwd_main<BF16, 6>(mq, mk, mv, mdo, mdq, mdk, mdv, p, st);
    case 7: return launch_bwd_main<BF16, 7>(mq, mk, mv, mdo, mdq, mdk, mdv, p, st);
    default: return launch_bwd_main<BF16, 8>(mq, mk, mv, mdo, mdq, mdk, mdv, p, st);
  }
}

template <bool BF16>
int run_bwd(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v, const kf_tensor4* o,
            const float* lse, const kf_tensor4* dout, const kf_tensor4* dq, const kf_tensor4* dk,
            const kf_tensor4* dv, float scale, int causal, void* workspace, size_t workspace_bytes,
            int32_t* status, cudaStream_t st) {
  const int B = (int)q->size[0], Hq = (int)q->size[1], Sq = (int)q->size[2], D = (int)q->size[3];
  const int Hkv = (int)k->size[1], Sk = (int)k->size[2];
  const int Sq_pad = (Sq + kBM - 1) / kBM * kBM;
  const int nqb = Sq_pad / kBM;
  const int nkb = (Sk + kBN - 1) / kBN;
  const int Sk_pad = nkb * kBN;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  float* dq_acc = reinterpret_cast<float*>(ws);
  const size_t acc_bytes = align256((size_t)B * Hq * nqb * D * kBM * 4);
  float* lse2 = reinterpret_cast<float*>(ws + acc_bytes);
  const size_t row_bytes = align256((size_t)B * Hq * Sq_pad * 4);
  float* delta = reinterpret_cast<float*>(ws + acc_bytes + row_bytes);
  const size_t kv_acc_bytes = align256((size_t)B * Hkv * Sk_pad * D * 4);
  float* dk_acc = reinterpret_cast<float*>(ws + acc_bytes + 2 * row_bytes);
  float* dv_acc = reinterpret_cast<float*>(ws + acc_bytes + 2 * row_bytes + kv_acc_bytes);

  // Query split of the key blocks; the parts need the dK/dV accumulators,
  // i.e. a workspace of kf_attn_bwd_workspace_bytes_kv bytes.
  //  * Causal problems with fewer key-block CTAs than two per SM (a long
  //    sequence sharded to one (batch, KV head) unit per GPU: key block 0
  //    sees every query block, the last one almost none, so one CTA per key
  //    block would leave the grid waiting on its heaviest CTA): parts target
  //    about six waves of equal CTAs (two waves measured 9-14% slower: the
  //    remainder parts and the last wave weigh less when the parts are
  //    smaller).
  //  * Non-causal problems with few key blocks: every key-block CTA has the
  //    same work, so what is lost is the last, partial wave of one CTA per
  //    SM (128 key blocks on 148 SMs keep 87% of them busy); the key blocks
  //    are cut into the number of parts (<= 16) that fills the waves best.
  const int sms = kf::sm_count_current_device();
  const int G = Hq / Hkv;
  int parts_max = 1, part_chunk = nqb;
  const size_t split_need = 256 + acc_bytes + 2 * row_bytes + 2 * kv_acc_bytes;
  const int64_t kb_ctas = (int64_t)B * Hkv * nkb;
  if (!causal && kb_ctas < 4 * (int64_t)sms && workspace_bytes >= split_need) {
    auto fill = [&](int64_t ctas) { return (double)ctas / (double)(((ctas + sms - 1) / sms) * sms); };
    double best_fill = fill(kb_ctas);
    for (int want = 2; want <= 16 && nqb / want >= 4; ++want) {
      const int chunk = (nqb + want - 1) / want;
      const int parts = (nqb + chunk - 1) / chunk;  // parts of `chunk` query blocks
      const double f = fill(kb_ctas * parts);
      if (f > best_fill + 0.02) {
        part_chunk = chunk;
        parts_max = parts;
        best_fill = f;
      }
    }
  }
  if (causal && kb_ctas < 2 * (int64_t)sms && workspace_bytes >= split_need) {
    int64_t total = 0;  // steps of the whole launch (query block x head per key block)
    for (int n = 0; n < nkb; ++n) total += (int64_t)G * (nqb - std::min((n * kBN) / kBM, nqb));
    total *= (int64_t)B * Hkv;
    const int64_t target = (total + 6 * sms - 1) / (6 * sms);
    part_chunk = (int)std::max<int64_t>(4, (target + G - 1) / G);
    parts_max = (nqb + part_chunk - 1) / part_chunk;
    if (parts_max <= 1) {
      parts_max = 1;
      part_chunk = nqb;
    }
  }
  const bool split = parts_max > 1;

  PrepArgs pa;
  pa.o = static_cast<const uint16_t*>(o->ptr);
  pa.dout = static_cast<const uint16_t*>(dout->ptr);
  pa.lse = lse;
  pa.lse2 = lse2;
  pa.delta = delta;
  for (int i = 0; i < 4; ++i) {
    pa.os[i] = o->stride[i];
    pa.dos[i] = dout->stride[i];
  }
  pa.Hq = Hq;
  pa.Sq = Sq;
  pa.Sq_pad = Sq_pad;
  pa.D = D;
  pa.rows = (int64_t)B * Hq * Sq_pad;
  pa.acc = reinterpret_cast<float4*>(dq_acc);
  pa.acc_vec4 = (int64_t)B * Hq * nqb * D * kBM / 4;
  pa.acc2 = split ? reinterpret_cast<float4*>(dk_acc) : nullptr;
  pa.acc2_vec4 = split ? (int64_t)(2 * kv_acc_bytes) / 16 : 0;
  const int64_t prep_blocks = std::min<int64_t>((pa.rows + 15) / 16, (int64_t)kf::sm_count_current_device() * 8);
  prep_kernel<BF16><<<(unsigned)std::max<int64_t>(prep_blocks, 1), 256, 0, st>>>(pa);
  int rc = kf::check_launch("kf_attn_bwd prep");
  if (rc) return rc;

  CUtensorMap mq, mk, mv, mdo, mdq, mdk, mdv;
  if ((rc = kf::encode_tmap_2d_f32(&mdq, dq_acc, (int64_t)B * Hq * nqb * D, kBM, 32, D))) return rc;
  if (split) {
    if ((rc = kf::encode_tmap_2d_f32(&mdk, dk_acc, (int64_t)B * Hkv * Sk_pad, D, 32, kBN))) return rc;
    if ((rc = kf::encode_tmap_2d_f32(&mdv, dv_acc, (int64_t)B * Hkv * Sk_pad, D, 32, kBN))) return rc;
  } else {
    mdk = mdq;  // unused without a split
    mdv = mdq;
  }
  if ((rc = kf::encode_tmap_4d(&mq, q, 64, kBM))) return rc;
  if ((rc = kf::encode_tmap_4d(&mdo, dout, 64, kBM))) return rc;
  if ((rc = kf::encode_tmap_4d(&mk, k, 64, kBN))) return rc;
  if ((rc = kf::encode_tmap_4d(&mv, v, 64, kBN))) return rc;

  BwdParams p;
  p.dk = static_cast<uint16_t*>(dk->ptr);
  p.dv = static_cast<uint16_t*>(dv->ptr);
  for (int i = 0; i < 4; ++i) {
    p.dks[i] = dk->stride[i];
    p.dvs[i] = dv->stride[i];
  }
  p.dq_acc = dq_acc;
  p.lse2 = lse2;
  p.delta = delta;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = Hq / Hkv;
  p.Sq = Sq;
  p.Sk = Sk;
  p.D = D;
  p.Sq_pad = Sq_pad;
  p.nqb = nqb;
  p.nkb = nkb;
  p.pairs_per_group = kPairsPerGroup;
  p.parts_max = parts_max;
  p.part_chunk = part_chunk;
  p.Sk_pad = Sk_pad;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * kLog2e;
  p.scale = scale;
  p.status = status;
  if ((rc = dispatch_bwd_main<BF16>((D + 15) / 16, mq, mk, mv, mdo, mdq, mdk, mdv, p, st))) return rc;
  if (split) {
    FinishKVArgs fk;
    fk.acc_k = dk_acc;
    fk.acc_v = dv_acc;
    fk.dk = static_cast<uint16_t*>(dk->ptr);
    fk.dv = static_cast<uint16_t*>(dv->ptr);
    for (int i = 0; i < 4; ++i) {
      fk.dks[i] = dk->stride[i];
      fk.dvs[i] = dv->stride[i];
    }
    fk.Hkv = Hkv;
    fk.Sk = Sk;
    fk.Sk_pad = Sk_pad;
    fk.D = D;
    fk.scale = scale;
    fk.rows = (int64_t)B * Hkv * Sk;
    const int64_t blocks = std::min<int64_t>((2 * fk.rows * (D / 8) + 255) / 256, (int64_t)sms * 8);
    finish_kv_kernel<BF16><<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, st>>>(fk);
    if ((rc = kf::check_launch("kf_attn_bwd finish dK/dV"))) return rc;
  }

  FinishArgs fa;
  fa.acc = dq_acc;
  fa.dq = static_cast<uint16_t*>(dq->ptr);
  for (int i = 0; i < 4; ++i) fa.qs[i] = dq->stride[i];
  fa.Hq = Hq;
  fa.Sq = Sq;
  fa.D = D;
  fa.nqb = nqb;
  fa.scale = scale;
  finish_kernel<BF16><<<dim3(nqb, B * Hq), 256, 0, st>>>(fa);
  return kf::check_launch("kf_attn_bwd finish");
}

}  // namespace

extern "C" size_t kf_attn_bwd_workspace_bytes(int64_t B, int64_t Hq, int64_t Sq, int64_t D) {
  const int64_t Sq_pad = (Sq + kBM - 1) / kBM * kBM;
  return 256 + align256((size_t)(B * Hq * Sq_pad) * D * 4) + 2 * align256((size_t)(B * Hq * Sq_pad) * 4);
}

extern "C" size_t kf_attn_bwd_workspace_bytes_kv(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk,
                                                 int64_t D) {
  const int64_t Sk_pad = (Sk + kBN - 1) / kBN * kBN;
  return kf_attn_bwd_workspace_bytes(B, Hq, Sq, D) + 2 * align256((size_t)(B * Hkv * Sk_pad) * D * 4);
}

extern "C" int kf_attn_bwd(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                           const kf_tensor4* o, const float* lse, const kf_tensor4* dout,
                           const kf_tensor4* dq, const kf_tensor4* dk, const kf_tensor4* dv,
                           int dtype, float scale, int causal, void* workspace,
                           size_t workspace_bytes, int32_t* status, void* stream) {
  using kf::set_error;
  if (!q || !k || !v || !o || !lse || !dout || !dq || !dk || !dv)
    return set_error(KF_ERR_INVALID, "kf_attn_bwd: null argument");
  if (dtype != KF_F16 && dtype != KF_BF16)
    return set_error(KF_ERR_INVALID, "kf_attn_bwd: dtype must be fp16 or bf16");
  const int64_t B = q->size[0], Hq = q->size[1], Sq = q->size[2], D = q->size[3];
  const int64_t Hkv = k->size[1], Sk = k->size[2];
  for (int i = 0; i < 4; ++i) {
    if (k->size[i] != v->size[i] || dk->size[i] != k->size[i] || dv->size[i] != k->size[i])
      return set_error(KF_ERR_INVALID, "kf_attn_bwd: K, V, dK and dV shapes must match");
    if (o->size[i] != q->size[i] || dout->size[i] != q->size[i] || dq->size[i] != q->size[i])
      return set_error(KF_ERR_INVALID, "kf_attn_bwd: O, dO and dQ must have Q's shape");
  }
  if (k->size[0] != B || k->size[3] != D)
    return set_error(KF_ERR_INVALID, "kf_attn_bwd: K/V batch and head_dim must match Q");
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Sk <= 0 || Hq % Hkv)
    return set_error(KF_ERR_INVALID, "kf_attn_bwd: bad dimensions or head grouping");
  if (D < 16 || D > 128 || D % 8)
    return set_error(KF_ERR_UNSUPPORTED, "kf_attn_bwd: head_dim must be a multiple of 8 in [16, 128]");
  if (Sq > (1 << 30) || Sk > (1 << 30) || B * Hq > 65535)
    return set_error(KF_ERR_UNSUPPORTED, "kf_attn_bwd: problem too large");
  for (const kf_tensor4* t : {q, k, v, o, dout, dq, dk, dv})
    if (!rows16(t))
      return set_error(KF_ERR_INVALID, "kf_attn_bwd: tensors need a contiguous last dim and 16-byte aligned rows");
  const size_t need = kf_attn_bwd_workspace_bytes(B, Hq, Sq, D);
  if (!workspace || workspace_bytes < need)
    return set_error(KF_ERR_WORKSPACE, "kf_attn_bwd: workspace needs %zu bytes", need);
  kf::DeviceGuard guard(q->ptr);
  if (guard.status()) return guard.status();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == KF_BF16)
    return run_bwd<true>(q, k, v, o, lse, dout, dq, dk, dv, scale, causal, workspace, workspace_bytes, status, st);
  return run_bwd<false>(q, k, v, o, lse, dout, dq, dk, dv, scale, causal, workspace, workspace_bytes, status, st);
}
