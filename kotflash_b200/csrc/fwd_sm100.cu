// K1: attention forward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces `_attention_fwd_kernel` (kotflash/kernels/triton_forward.py:21-165)
// and its launcher `attention_forward` (triton_forward.py:372-456).  Computes
// O = softmax(scale * Q K^T + mask) V and the row LSE (natural log) for
// upper-left causal or full masks, GQA/MQA head mapping, fp16/bf16,
// 16 <= D <= 128 (D % 8 == 0; columns past D are zero-filled by TMA).
//
// CTA = two 128-row Q tiles that share one KV head (two heads of the same
// GQA group at the same rows, or two consecutive row blocks of one head),
// so every K/V tile fetched by TMA feeds both.  Warp roles:
//   warps 0-3  softmax for tile 0   (thread t owns query row t = TMEM lane t)
//   warps 4-7  softmax for tile 1
//   warp  8    TMA producer (Q once, then K/V blocks of BN keys)
//   warp  9    TMEM allocator + tcgen05.mma issuer for tile 0
//   warp 10    tcgen05.mma issuer for tile 1
//   warp 11    spare (completes the third warpgroup)
// The softmax warpgroups raise their register limit to 224 (setmaxnreg) and
// warps 8-11 lower theirs to 56.
//
// Each tile has its own score buffer S, probability buffer P (16-bit) and
// output accumulator O in tensor memory (512 columns):
//   head_dim <= 64  (BN 128): S0 [0,128)  P0 [128,192)  O0 [192,256)  S1 [256,384)  P1 [384,448)  O1 [448,512)
//   head_dim 65-96  (BN  96): S0 [0,96)   P0 [96,144)   O0 [160,256)  S1 [256,352)  P1 [352,400)  O1 [416,512)
//   head_dim 97-128 (BN  80): S0 [0,80)   P0 [80,120)   O0 [128,256)  S1 [256,336)  P1 [336,376)  O1 [384,512)
// Because P does not overlay S, a tile's softmax releases S as soon as it has
// loaded the scores into registers, and the tile's issuer computes the next
// block's S = Q K^T while the softmax still works on this block; P feeds the
// O += P V product straight from tensor memory (A operand in TMEM).  Per tile
// and block j the issuer runs
//   [S(j) loaded]  S(j+1) = Q K_{j+1}^T      [P(j) stored]  O += P(j) V_j
// so the softmax of a tile runs block after block without waiting for its own
// GEMMs, and the two tiles' GEMMs fill the tensor pipe between them.  With
// P over S (an earlier layout) each tile's chain was softmax + its two GEMMs
// in series, and the tensor pipe sat idle about half the time.  The block
// width is the widest multiple of 16 for which a tile's S and P fit below its
// O in 256 columns (80 + 40 + 128 at head_dim 128, 96 + 48 + 96 at head_dim
// 96); fewer keys per block cost a little shared-memory bandwidth per FLOP
// and more per-block synchronisation.
// Two issuing threads matter on sm_100: the tensor pipe holds almost no
// queued MMAs, so every cycle an issuing thread spends on an mbarrier wait, a
// tcgen05 fence or a commit would idle the pipe; with one issuer per tile,
// the other tile's MMAs fill those gaps.  The running max is only raised (and
// O rescaled) when it grows by more than 2^8, so most blocks skip the O round
// trip; P stays <= 256, which fp16/bf16 hold exactly enough.  The softmax
// computes its exponentials partly on the MUFU unit and partly as a
// polynomial on the fp32 pipe (packed f32x2 arithmetic), because 16 MUFU
// results per clock per SM alone cannot keep up with the tensor cores at
// head_dim 128.  At the end of an item each softmax warp stages its rows of
// O (16 rows x 64 columns at a time, 16-bit, 128-byte swizzle) in its own
// 2 KB of shared memory and one lane writes them with a TMA store.
// Shared memory: Q tiles [2][NP][128][64], K and V rings [STAGES][NP][BN][64],
// the eight 2 KB staging areas, then the barriers.
#include <math.h>

#include <algorithm>

#include "kf_host.h"
#include "kf_sm100.cuh"

namespace {

constexpr int kBlockM = 128;
constexpr int kThreads = 384;  // 3 warpgroups: two softmax, one producer + MMA issuers + spare
// Register split between the warpgroups (setmaxnreg): a softmax thread holds a
// 128-column score row and its packed probabilities, the other roles little.
// 256 * 224 + 128 * 56 = 384 * 168, the allocation the block launches with.
constexpr int kRegSoftmax = 224, kRegOther = 56;
constexpr int kMaxStages = 4;  // deepest K/V ring (kv_stages)
// Epilogue staging: each softmax warp packs 16 rows x 64 columns of O (2 KB,
// 128-byte swizzle) in shared memory and hands them to one TMA store.
constexpr int kStoreRows = 16;
constexpr int kStageBytes = kStoreRows * 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Of every 8 exponential pairs in an unmasked block, this many run as the
// fp32-pipe polynomial and the rest on MUFU.
// (1 and 3 of 8 measured no faster with the early-release schedule)
#ifndef KF_FWD_POLY_PAIRS
#define KF_FWD_POLY_PAIRS 2
#endif
constexpr int kPolyPairs = KF_FWD_POLY_PAIRS;


struct FwdParams {
  uint16_t* o;
  float* lse;
  int64_t os[4];
  int B, Hq, Hkv, G, Sq, Sk, D;
  int causal;
  int m_blocks;        // cdiv(Sq, 128)
  int slots_per_kvh;   // G * m_blocks
  int ctas_per_kvh;    // cdiv(slots_per_kvh, 2): work items per KV head
  int n_items;         // B * Hkv * ctas_per_kvh
  float scale_log2;
  int32_t* status;
};

// Keys per K/V block, K/V ring depth and TMEM columns of each tile's S, P and
// O for a head dim of KS * 16 (layouts above).  Tile t owns columns
// [256 t, 256 t + 256): S at the bottom, P right above it, O at the top
// (its width rounded up to 32 columns).  The block width is the widest
// multiple of 16 whose S and P fit below O.  (A layout with S and P of both
// tiles in the low 256 columns and both O in the high 256 measured the same
// at head_dim 128 and 2-5% slower at 72 and 96, interleaved in one process.)
__host__ __device__ constexpr int block_n(int ks) { return ks > 6 ? 80 : (ks > 4 ? 96 : 128); }
__host__ __device__ constexpr int kv_stages(int ks) { return ks > 4 ? 3 : 4; }
__host__ __device__ constexpr int o_width(int ks) { return (ks * 16 + 31) / 32 * 32; }
__host__ __device__ constexpr uint32_t s_col_of(int ks, int t) { return 256u * t + 0u * ks; }
__host__ __device__ constexpr uint32_t p_col_of(int ks, int t) { return 256u * t + block_n(ks); }
__host__ __device__ constexpr uint32_t o_col_of(int ks, int t) { return 256u * t + 256u - o_width(ks); }
// The six buffers of a layout are disjoint and inside the 512 columns.
__host__ __device__ constexpr bool disjoint(uint32_t a, uint32_t an, uint32_t b, uint32_t bn) {
  return a + an <= b || b + bn <= a;
}
__host__ __device__ constexpr bool layout_ok(int ks) {
  const uint32_t bn = block_n(ks), w[3] = {bn, bn / 2, (uint32_t)o_width(ks)};
  uint32_t c[6] = {s_col_of(ks, 0), p_col_of(ks, 0), o_col_of(ks, 0),
                   s_col_of(ks, 1), p_col_of(ks, 1), o_col_of(ks, 1)};
  for (int i = 0; i < 6; ++i) {
    if (c[i] + w[i % 3] > 512u) return false;
    for (int j = i + 1; j < 6; ++j)
      if (!disjoint(c[i], w[i % 3], c[j], w[j % 3])) return false;
  }
  return true;
}
static_assert(layout_ok(1) && layout_ok(2) && layout_ok(3) && layout_ok(4) && layout_ok(5) &&
                  layout_ok(6) && layout_ok(7) && layout_ok(8),
              "TMEM layout");

struct __align__(8) FwdBarriers {
  uint64_t q_full, q_empty;
  uint64_t k_full[kMaxStages], k_empty[kMaxStages];
  uint64_t v_full[kMaxStages], v_empty[kMaxStages];
  uint64_t s_full[2], s_free[2], p_full[2], pv_done[2];
  uint64_t o_final[2];
  uint64_t turn[2];  // exponential phases of the two tiles alternate
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, FwdBarriers* bars,
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

// Work item of a CTA: KV head (b, kvh) and up to two (head, row0) tiles.
struct TileInfo {
  int b, kvh;
  int head[2], row0[2];
  int valid[2];
  int n_blocks;
};

// Items are numbered heaviest first across all KV heads (for causal masks the
// later row blocks see more keys).  The persistent CTAs take them in rounds
// of gridDim.x items, in forward order on even rounds and reverse order on
// odd rounds, so a CTA that drew a heavy item in one round draws a light one
// in the next and the CTAs' totals stay close.
template <int BN>
__device__ __forceinline__ TileInfo tile_info(const FwdParams& p, int item) {
  TileInfo ti;
  const int per_bh = p.ctas_per_kvh;
  const int n_bh = p.B * p.Hkv;
  const int bh = item % n_bh;
  const int c = per_bh - 1 - item / n_bh;
  ti.b = bh / p.Hkv;
  ti.kvh = bh % p.Hkv;
  int row_end_max = 0;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int slot = 2 * c + t;
    ti.valid[t] = slot < p.slots_per_kvh;
    const int s = ti.valid[t] ? slot : 2 * c;
    const int mb = s / p.G, g = s % p.G;
    ti.head[t] = ti.kvh * p.G + g;
    ti.row0[t] = mb * kBlockM;
    if (ti.valid[t]) row_end_max = max(row_end_max, min(ti.row0[t] + kBlockM, p.Sq));
  }
  const int key_end = p.causal ? min(p.Sk, row_end_max) : p.Sk;
  ti.n_blocks = (key_end + BN - 1) / BN;
  return ti;
}

// Item of round r for this CTA, or -1 when the last round has none for it.
__device__ __forceinline__ int round_item(int r, int n_items) {
  const int g = (int)gridDim.x;
  const int idx = r * g + ((r & 1) ? g - 1 - (int)blockIdx.x : (int)blockIdx.x);
  return idx < n_items ? idx : -1;
}

template <bool BF16, int NP, int KS>
__global__ void __launch_bounds__(kThreads, 1)
fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
           const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
           const FwdParams p) {
  constexpr int BN = block_n(KS);             // keys per K/V block
  constexpr int STAGES = kv_stages(KS);       // K/V ring depth
  constexpr int QPANEL = kBlockM * 128;       // bytes of one 64-column panel of a 128-row Q tile
  constexpr int QTILE = NP * QPANEL;
  constexpr int KPANEL = BN * 128;            // one 64-column panel of a K or V block
  constexpr int KTILE = NP * KPANEL;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                          // [2][NP][128][64]
  uint8_t* sK = sQ + 2 * QTILE;                // [STAGES][NP][BN][64]
  uint8_t* sV = sK + STAGES * KTILE;           // [STAGES][NP][BN][64]
  uint8_t* sE = sV + STAGES * KTILE;           // [8 softmax warps][kStoreRows][64] epilogue staging
  FwdBarriers* bars = reinterpret_cast<FwdBarriers*>(sE + 8 * kStageBytes);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int d_pad16 = KS * 16;  // head dim rounded up to the MMA K step

  if (tid == 0) {
    kf::mbar_init(&bars->q_full, 1);
    kf::mbar_init(&bars->q_empty, 2);  // one commit per issuer
    for (int s = 0; s < STAGES; ++s) {
      kf::mbar_init(&bars->k_full[s], 1);
      kf::mbar_init(&bars->k_empty[s], 2);
      kf::mbar_init(&bars->v_full[s], 1);
      kf::mbar_init(&bars->v_empty[s], 2);
    }
    for (int t = 0; t < 2; ++t) {
      kf::mbar_init(&bars->s_full[t], 1);
      kf::mbar_init(&bars->s_free[t], 128);
      kf::mbar_init(&bars->p_full[t], 128);
      kf::mbar_init(&bars->pv_done[t], 1);
      kf::mbar_init(&bars->o_final[t], 1);
      kf::mbar_init(&bars->turn[t], 128);
    }
    bars->abort_flag = 0;
    kf::fence_barrier_init();
  }
  if (warp == 9) {
    kf::tmem_alloc(&bars->tmem_base, 512);
    kf::tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    kf::tma_prefetch_desc(&map_q);
    kf::tma_prefetch_desc(&map_k);
    kf::tma_prefetch_desc(&map_v);
    kf::tma_prefetch_desc(&map_o);
  }
  kf::tc_fence_before();
  __syncthreads();
  kf::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // Persistent CTA: every role walks the same item sequence (round_item);
  // barrier phases run on across items (g counts K/V blocks of all items,
  // it counts items, jt counts a tile's blocks).
  const int rounds = (p.n_items + (int)gridDim.x - 1) / (int)gridDim.x;
  if (warp >= 8) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegOther));
   if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int g = 0, it = 0;
      for (int rd = 0; rd < rounds; ++rd) {
        const int item = round_item(rd, p.n_items);
        if (item < 0) continue;
        const TileInfo ti = tile_info<BN>(p, item);
        const int nt = ti.valid[1] ? 2 : 1;
        // the previous item's last QK^T has read the Q tiles
        if (it > 0 && !wait_bar(&bars->q_empty, (it - 1) & 1, bars, p.status)) break;
        kf::mbar_arrive_expect_tx(&bars->q_full, nt * QTILE);
#pragma unroll
        for (int t = 0; t < 2; ++t)
          if (t < nt)
#pragma unroll
            for (int pn = 0; pn < NP; ++pn)
              kf::tma_load_4d(sQ + t * QTILE + pn * QPANEL, &map_q, &bars->q_full, pn * 64, ti.row0[t],
                              ti.head[t], ti.b);
        bool ok = true;
        for (int j = 0; j < ti.n_blocks; ++j) {
          const int gj = g + j;
          const int s = gj % STAGES;
          const uint32_t ph = ((gj / STAGES) & 1) ^ 1;
          if (!(ok = wait_bar(&bars->k_empty[s], ph, bars, p.status))) break;
          kf::mbar_arrive_expect_tx(&bars->k_full[s], KTILE);
#pragma unroll
          for (int pn = 0; pn < NP; ++pn)
            kf::tma_load_4d(sK + s * KTILE + pn * KPANEL, &map_k, &bars->k_full[s], pn * 64, j * BN, ti.kvh,
                            ti.b);
          if (!(ok = wait_bar(&bars->v_empty[s], ph, bars, p.status))) break;
          kf::mbar_arrive_expect_tx(&bars->v_full[s], KTILE);
#pragma unroll
          for (int pn = 0; pn < NP; ++pn)
            kf::tma_load_4d(sV + s * KTILE + pn * KPANEL, &map_v, &bars->v_full[s], pn * 64, j * BN, ti.kvh,
                            ti.b);
        }
        if (!ok) break;
        g += ti.n_blocks;
        ++it;
      }
    }
  } else if (warp == 9 || warp == 10) {
    // ------------------------------------------------------------ MMA issuers
    const int t = warp - 9;  // this thread issues every MMA of Q tile t
    if (lane == 0) {
      const uint32_t idesc_qk = kf::make_idesc_f16(BF16, kBlockM, BN, 0, 0);
      const uint32_t idesc_pv = kf::make_idesc_f16(BF16, kBlockM, d_pad16, 0, 1);
      // Descriptors are built once; each MMA only adds a compile-time offset
      // to the low word of a base descriptor.
      const kf::SDesc dq = kf::make_sdesc_split(kf::smem_u32(sQ + t * QTILE), 16, 1024);
      const kf::SDesc dk = kf::make_sdesc_split(kf::smem_u32(sK), 16, 1024);
      const kf::SDesc dv = kf::make_sdesc_split(kf::smem_u32(sV), KPANEL, 1024);
      const uint32_t s_tm = tmem + s_col_of(KS, t), p_tm = tmem + p_col_of(KS, t), o_tm = tmem + o_col_of(KS, t);
      // Each GEMM is one straight-line run of MMAs (compile-time trip counts).
      auto issue_qk = [&](int gj) {
        const uint32_t koff = (gj % STAGES) * KTILE;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk)
          kf::umma_ss(s_tm, kf::sdesc_at_here(dq, (kk >> 2) * QPANEL + (kk & 3) * 32),
                      kf::sdesc_at_here(dk, koff + (kk >> 2) * KPANEL + (kk & 3) * 32), idesc_qk, kk > 0);
      };
      auto issue_pv = [&](int gj, bool first) {
        const uint32_t voff = (gj % STAGES) * KTILE;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          kf::umma_ts(o_tm, p_tm + kk * 8, kf::sdesc_at_here(dv, voff + kk * 2048), idesc_pv,
                      (!first || kk > 0));
      };
      int g = 0, it = 0, jt = 0;  // K/V blocks (all items), items, blocks of tile t
      bool ok = true;
      for (int rd = 0; ok && rd < rounds; ++rd) {
        const int item = round_item(rd, p.n_items);
        if (item < 0) continue;
        const TileInfo ti = tile_info<BN>(p, item);
        const int nt = ti.valid[1] ? 2 : 1;
        const int nblk = ti.n_blocks;
        if (t < nt) {
          // With one Q tile the tile-0 issuer commits twice to the barriers
          // both issuers release, so their arrival counts stay fixed.
          const int rel = nt == 2 ? 1 : 2;
          auto release = [&](uint64_t* bar) {
            for (int k = 0; k < rel; ++k) kf::umma_commit(bar);
          };
          ok = wait_bar(&bars->q_full, it & 1, bars, p.status) &&
               wait_bar(&bars->k_full[g % STAGES], (g / STAGES) & 1, bars, p.status);
          if (!ok) break;
          kf::tc_fence_after();
          issue_qk(g);
          kf::umma_commit(&bars->s_full[t]);
          if (nblk == 1) release(&bars->q_empty);
          release(&bars->k_empty[g % STAGES]);
          for (int j = 0; j < nblk; ++j) {
            const int gj = g + j;
            if (j + 1 < nblk) {
              // S(j) is in the softmax's registers: compute S(j+1) now
              const int s1 = (gj + 1) % STAGES;
              if (!(ok = wait_bar(&bars->s_free[t], (jt + j) & 1, bars, p.status))) break;
              if (!(ok = wait_bar(&bars->k_full[s1], ((gj + 1) / STAGES) & 1, bars, p.status))) break;
              kf::tc_fence_after();
              issue_qk(gj + 1);
              kf::umma_commit(&bars->s_full[t]);
              if (j + 2 == nblk) release(&bars->q_empty);  // last QK^T of the item
              release(&bars->k_empty[s1]);
            }
            const int s = gj % STAGES;
            if (!(ok = wait_bar(&bars->v_full[s], (gj / STAGES) & 1, bars, p.status))) break;
            if (!(ok = wait_bar(&bars->p_full[t], (jt + j) & 1, bars, p.status))) break;
            kf::tc_fence_after();
            issue_pv(gj, j == 0);
            kf::umma_commit(&bars->pv_done[t]);
            release(&bars->v_empty[s]);
          }
          kf::umma_commit(&bars->o_final[t]);
          jt += nblk;
        }
        g += nblk;
        ++it;
      }
    }
   }
   // warp 11 is spare: it completes the third warpgroup for the register split
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegSoftmax));
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;        // tile handled by this warpgroup
    const int r = (warp & 3) * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t s_col = s_col_of(KS, t), p_col = p_col_of(KS, t), o_col = o_col_of(KS, t);
    int jt = 0, vt = 0, jturn = 0;  // blocks of tile t, items of tile t, blocks of two-tile items
    bool ok = true;
    for (int rd = 0; ok && rd < rounds; ++rd) {
      const int item = round_item(rd, p.n_items);
      if (item < 0) continue;
      const TileInfo ti = tile_info<BN>(p, item);
      const int nt = ti.valid[1] ? 2 : 1;
      const int nblk = ti.n_blocks;
      // this warpgroup's tile, selected without indexing the arrays by a
      // run-time value (which would put TileInfo in local memory)
      const bool my_valid = t ? ti.valid[1] : ti.valid[0];
      const int my_row0 = t ? ti.row0[1] : ti.row0[0];
      const int my_head = t ? ti.head[1] : ti.head[0];
      if (!my_valid) continue;
      const int row = my_row0 + r;
      float m_ref = -INFINITY, l_sum = 0.f;
      for (int j = 0; ok && j < nblk; ++j) {
        if (!(ok = __all_sync(0xffffffffu, wait_bar(&bars->s_full[t], (jt + j) & 1, bars, p.status)))) break;
        kf::tc_fence_after();
        uint32_t sr[BN];
        kf::tmem_ld32(lane_base + s_col + 0, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        kf::tmem_ld32(lane_base + s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        if constexpr (BN == 128) {
          kf::tmem_ld32(lane_base + s_col + 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
          kf::tmem_ld32(lane_base + s_col + 96, *reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
        } else if constexpr (BN == 96) {
          kf::tmem_ld32(lane_base + s_col + 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
        } else {
          static_assert(BN == 80, "block width");
          kf::tmem_ld16(lane_base + s_col + 64, *reinterpret_cast<uint32_t(*)[16]>(&sr[64]));
        }
        kf::tmem_wait_ld();
        // the scores are in registers: the issuer may overwrite S with the next block's
        kf::tc_fence_before();
        kf::mbar_arrive(&bars->s_free[t]);
        const int key0 = j * BN;
        const bool need_mask = (key0 + BN > p.Sk) || (p.causal && key0 + BN - 1 > my_row0);
        if (need_mask) {
          const int lim = min(p.Sk - key0, p.causal ? row - key0 + 1 : BN);
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c >= lim) sr[c] = 0xFF800000u;  // -inf
        }
        // Row max of the raw scores (the scale is positive, so it commutes),
        // four independent chains of three-input maxima.
        float mx;
        {
          float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll
          for (int c = 0; c < BN; c += 8) {
            a0 = kf::fmax3(a0, __uint_as_float(sr[c + 0]), __uint_as_float(sr[c + 1]));
            a1 = kf::fmax3(a1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
            a2 = kf::fmax3(a2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
            a3 = kf::fmax3(a3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
          }
          mx = kf::fmax3(a0, a1, fmaxf(a2, a3)) * p.scale_log2;
        }
        float alpha = 1.f;
        bool rescale_o = false;
        if (j == 0) {
          m_ref = mx;
        } else if (mx > m_ref + kRescaleThreshold) {
          alpha = kf::ex2(m_ref - mx);
          m_ref = mx;
          rescale_o = true;
        }
        const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
        l_sum *= alpha;
        // Tile 0 exponentiates block j after tile 1 finished block j-1, tile 1
        // after tile 0 finished block j: the two warps sharing each SM
        // sub-partition never compete for MUFU and issue slots.
        if (nt == 2 && (t == 1 || j > 0)) {
          if (!(ok = wait_bar(&bars->turn[t], (jturn + j - (t == 1 ? 0 : 1)) & 1, bars, p.status))) break;
        }
        // P = 2^(s * scale_log2 - m): the argument is one packed fma per pair;
        // masked blocks (-inf entries) use MUFU only, full blocks send
        // kPolyPairs of every 8 pairs to the fp32-pipe polynomial.
        const uint64_t scl = kf::f2(p.scale_log2, p.scale_log2), negm = kf::f2(-m_use, -m_use);
        uint32_t pk[BN / 2];
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < BN / 2; ++c) {
            float x0, x1;
            kf::f2_split(kf::fma2(kf::f2(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])), scl, negm), x0, x1);
            const float p0 = kf::ex2(x0), p1 = kf::ex2(x1);
            acc[c & 3] = kf::add2(acc[c & 3], kf::f2(p0, p1));
            pk[c] = kf::pack2<BF16>(p0, p1);
          }
        } else {
#pragma unroll
          for (int c = 0; c < BN / 2; ++c) {
            float x0, x1;
            kf::f2_split(kf::fma2(kf::f2(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])), scl, negm), x0, x1);
            const uint64_t pp = (c & 7) < kPolyPairs ? kf::exp2_poly2(x0, x1) : kf::f2(kf::ex2(x0), kf::ex2(x1));
            acc[c & 3] = kf::add2(acc[c & 3], pp);
            float p0, p1;
            kf::f2_split(pp, p0, p1);
            pk[c] = kf::pack2<BF16>(p0, p1);
          }
        }
        {
          float s0, s1;
          kf::f2_split(kf::add2(kf::add2(acc[0], acc[1]), kf::add2(acc[2], acc[3])), s0, s1);
          l_sum += s0 + s1;
        }
        if (nt == 2) kf::mbar_arrive(&bars->turn[t ^ 1]);
        // P(j) goes where P(j-1) was and O may be rescaled: both need the
        // previous block's O += P V to have completed
        if (j > 0) {
          if (!(ok = __all_sync(0xffffffffu, wait_bar(&bars->pv_done[t], (jt + j - 1) & 1, bars, p.status)))) break;
          kf::tc_fence_after();
        }
        kf::tmem_st32(lane_base + p_col + 0, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
        if constexpr (BN == 128) {
          kf::tmem_st32(lane_base + p_col + 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
        } else if constexpr (BN == 96) {
          kf::tmem_st16(lane_base + p_col + 32, *reinterpret_cast<const uint32_t(*)[16]>(&pk[32]));
        } else {
          kf::tmem_st8(lane_base + p_col + 32, *reinterpret_cast<const uint32_t(*)[8]>(&pk[32]));
        }
        if (__any_sync(0xffffffffu, rescale_o)) {
          // O row *= alpha (alpha == 1 on rows that keep their reference max)
          for (int c0 = 0; c0 < d_pad16; c0 += 32) {
            uint32_t orow[32];
            kf::tmem_ld32(lane_base + o_col + c0, orow);
            kf::tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) orow[c] = __float_as_uint(__uint_as_float(orow[c]) * alpha);
            kf::tmem_st32(lane_base + o_col + c0, orow);
          }
        }
        kf::tmem_wait_st();
        kf::tc_fence_before();
        kf::mbar_arrive(&bars->p_full[t]);
      }
      // -------------------------------------------------------- epilogue
      // O is read from TMEM before this thread's next p_full arrival, which
      // is what lets the next item's first PV overwrite it.  Rows leave
      // through TMA stores of 16 rows x 64 columns staged in shared memory
      // (one row per thread, 128-byte swizzle: 16-byte chunk c of staging row
      // r sits at chunk c ^ (r & 7)); the store clips rows past Sq and
      // columns past D.
      if (ok && (ok = __all_sync(0xffffffffu, wait_bar(&bars->o_final[t], vt & 1, bars, p.status)))) {
        kf::tc_fence_after();
        const float inv_l = l_sum > 0.f ? 1.f / l_sum : 0.f;
        uint8_t* stage = sE + warp * kStageBytes;
        const int srow = lane & (kStoreRows - 1);
        const int row_base = my_row0 + (warp & 3) * 32;
#pragma unroll
        for (int c0 = 0; c0 < d_pad16; c0 += 64) {
          uint32_t ov[64];
          kf::tmem_ld32(lane_base + o_col + c0, *reinterpret_cast<uint32_t(*)[32]>(&ov[0]));
          if (c0 + 32 < d_pad16) {
            kf::tmem_ld32(lane_base + o_col + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&ov[32]));
          } else {
#pragma unroll
            for (int c = 32; c < 64; ++c) ov[c] = 0u;
          }
          kf::tmem_wait_ld();
          uint32_t pk[32];
#pragma unroll
          for (int c = 0; c < 32; ++c)
            pk[c] = kf::pack2<BF16>(__uint_as_float(ov[2 * c]) * inv_l, __uint_as_float(ov[2 * c + 1]) * inv_l);
#pragma unroll
          for (int half = 0; half < 32 / kStoreRows; ++half) {
            // the previous store of this warp has read the staging rows
            if (lane == 0) kf::bulk_wait_group_read<0>();
            __syncwarp();
            if (lane / kStoreRows == half) {
#pragma unroll
              for (int ch = 0; ch < 8; ++ch)
                *reinterpret_cast<uint4*>(stage + srow * 128 + ((ch ^ (srow & 7)) << 4)) =
                    make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
            }
            kf::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              kf::tma_store_4d(&map_o, stage, c0, row_base + half * kStoreRows, my_head, ti.b);
              kf::bulk_commit_group();
            }
          }
        }
        if (row < p.Sq)
          p.lse[((int64_t)ti.b * p.Hq + my_head) * p.Sq + row] =
              l_sum > 0.f ? (m_ref + log2f(l_sum)) * kLn2 : -INFINITY;
      }
      jt += nblk;
      ++vt;
      if (nt == 2) jturn += nblk;
    }
    // this warp's last O stores have written global memory
    if (lane == 0) kf::bulk_wait_group<0>();
    __syncwarp();
  }

  kf::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    kf::tc_fence_after();
    kf::tmem_dealloc(tmem, 512);
  }
}

bool rows16(const kf_tensor4* t) {
  if (!t || !kf::aligned16(t->ptr) || t->stride[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (t->size[i] > 1 && (t->stride[i] % 8) != 0) return false;
  return true;
}

template <bool BF16, int KS>
int launch_fwd(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
               const FwdParams& p, cudaStream_t st) {
  constexpr int NP = KS > 4 ? 2 : 1;
  constexpr size_t QTILE = (size_t)NP * kBlockM * 128;
  constexpr size_t KTILE = (size_t)NP * block_n(KS) * 128;
  const size_t smem = 1024 + 2 * QTILE + 2 * (size_t)kv_stages(KS) * KTILE + 8 * (size_t)kStageBytes +
                      sizeof(FwdBarriers);
  auto kern = fwd_kernel<BF16, NP, KS>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return kf::set_error(KF_ERR_CUDA, "kf_attn_fwd: cannot reserve %zu bytes of shared memory", smem);
  // setmaxnreg.inc waits until the block's launch allocation covers the
  // split, so refuse to launch if the compiler allocated less than that.
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess ||
      fa.numRegs * kThreads < 256 * kRegSoftmax + 128 * kRegOther)
    return kf::set_error(KF_ERR_CUDA, "kf_attn_fwd: register split does not fit (%d registers)", fa.numRegs);
  // A CTA that walks several items must not meet a single-tile item before a
  // two-tile one: the tile-1 issuer skips a single-tile item without waiting,
  // so at the next item its parity waits on the Q and K/V barriers could run
  // two phases ahead of the producer and return at once.  Single-tile items
  // (an odd slot count per KV head) are the first n_bh of the item order, so
  // a launch that has them and more items than SMs gives every CTA one item.
  const int sms = kf::sm_count_current_device();
  const bool single_tile_items = (p.slots_per_kvh & 1) != 0;
  const int grid = (single_tile_items && p.n_items > sms) ? p.n_items : std::min(p.n_items, sms);
  kern<<<(unsigned)grid, kThreads, smem, st>>>(mq, mk, mv, mo, p);
  return kf::check_launch("kf_attn_fwd");
}

template <bool BF16>
int dispatch_fwd(int ks, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                 const CUtensorMap& mo, const FwdParams& p, cudaStream_t st) {
  switch (ks) {
    case 1: return launch_fwd<BF16, 1>(mq, mk, mv, mo, p, st);
    case 2: return launch_fwd<BF16, 2>(mq, mk, mv, mo, p, st);
    case 3: return launch_fwd<BF16, 3>(mq, mk, mv, mo, p, st);
    case 4: return launch_fwd<BF16, 4>(mq, mk, mv, mo, p, st);
    case 5: return launch_fwd<BF16, 5>(mq, mk, mv, mo, p, st);
    case 6: return launch_fwd<BF16, 6>(mq, mk, mv, mo, p, st);
    case 7: return launch_fwd<BF16, 7>(mq, mk, mv, mo, p, st);
    default: return launch_fwd<BF16, 8>(mq, mk, mv, mo, p, st);
  }
}

}  // namespace

extern "C" int kf_attn_fwd(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                           const kf_tensor4* o, float* lse, int dtype, float scale, int causal,
                           int32_t* status, void* stream) {
  using kf::set_error;
  if (!q || !k || !v || !o || !lse) return set_error(KF_ERR_INVALID, "kf_attn_fwd: null argument");
  if (dtype != KF_F16 && dtype != KF_BF16)
    return set_error(KF_ERR_INVALID, "kf_attn_fwd: dtype must be fp16 or bf16");
  const int64_t B = q->size[0], Hq = q->size[1], Sq = q->size[2], D = q->size[3];
  const int64_t Hkv = k->size[1], Sk = k->size[2];
  for (int i = 0; i < 4; ++i) {
    if (k->size[i] != v->size[i]) return set_error(KF_ERR_INVALID, "kf_attn_fwd: K and V shapes must match");
    if (o->size[i] != q->size[i]) return set_error(KF_ERR_INVALID, "kf_attn_fwd: O must have Q's shape");
  }
  if (k->size[0] != B || k->size[3] != D)
    return set_error(KF_ERR_INVALID, "kf_attn_fwd: K/V batch and head_dim must match Q");
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Sk <= 0)
    return set_error(KF_ERR_INVALID, "kf_attn_fwd: dimensions must be non-zero");
  if (Hq % Hkv) return set_error(KF_ERR_INVALID, "kf_attn_fwd: Hq must be divisible by Hkv");
  if (D < 16 || D > 128 || D % 8)
    return set_error(KF_ERR_UNSUPPORTED, "kf_attn_fwd: head_dim must be a multiple of 8 in [16, 128]");
  if (Sq > (1 << 30) || Sk > (1 << 30) || B > 65535 || Hq > 65535)
    return set_error(KF_ERR_UNSUPPORTED, "kf_attn_fwd: problem too large");
  if (!rows16(q) || !rows16(k) || !rows16(v) || !rows16(o))
    return set_error(KF_ERR_INVALID, "kf_attn_fwd: tensors need a contiguous last dim and 16-byte aligned rows");

  kf::DeviceGuard guard(q->ptr);
  if (guard.status()) return guard.status();
  const int box_inner = 64;
  CUtensorMap mq, mk, mv, mo;
  int rc;
  if ((rc = kf::encode_tmap_4d(&mq, q, box_inner, kBlockM))) return rc;
  const int bn = block_n((int)((D + 15) / 16));
  if ((rc = kf::encode_tmap_4d(&mk, k, box_inner, bn))) return rc;
  if ((rc = kf::encode_tmap_4d(&mv, v, box_inner, bn))) return rc;
  if ((rc = kf::encode_tmap_4d(&mo, o, box_inner, kStoreRows))) return rc;

  FwdParams p;
  p.o = static_cast<uint16_t*>(o->ptr);
  p.lse = lse;
  for (int i = 0; i < 4; ++i) p.os[i] = o->stride[i];
  p.B = (int)B;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.G = (int)(Hq / Hkv);
  p.Sq = (int)Sq;
  p.Sk = (int)Sk;
  p.D = (int)D;
  p.causal = causal ? 1 : 0;
  p.m_blocks = (int)((Sq + kBlockM - 1) / kBlockM);
  p.slots_per_kvh = p.G * p.m_blocks;
  p.ctas_per_kvh = (p.slots_per_kvh + 1) / 2;
  p.n_items = (int)((int64_t)p.B * p.Hkv * p.ctas_per_kvh);
  p.scale_log2 = scale * kLog2e;
  p.status = status;
  if ((int64_t)p.B * p.Hkv * p.ctas_per_kvh > 0x7fffffffLL)
    return set_error(KF_ERR_UNSUPPORTED, "kf_attn_fwd: grid too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int ks = (int)((D + 15) / 16);
  return dtype == KF_BF16 ? dispatch_fwd<true>(ks, mq, mk, mv, mo, p, st)
                          : dispatch_fwd<false>(ks, mq, mk, mv, mo, p, st);
}
