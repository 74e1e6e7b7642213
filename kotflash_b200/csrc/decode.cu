// K3: split-KV decode for short queries (Sq <= 16) over long, possibly strided
// K/V, plus K3b, the LSE-weighted merge of split partials.
//
// Replaces the reference's `_attention_fwd_split_kv` + `_attention_fwd_split_kv_reduce`
// (kotflash/kernels/triton_forward.py:170-349), `_strided_decode_split` +
// `_strided_decode_reduce` (kotflash/kernels/triton_decode.py:17-104, 242-297)
// and the fused one-token append `_strided_decode_append_split`
// (triton_decode.py:109-238).
//
// Design (HBM-bound):
//  * one CTA per (split, batch, KV head, row block): all GROUP x Sq query rows
//    that share a KV head are packed into one tile, so each K/V byte of the
//    split is read from HBM exactly once (the reference reads it once per
//    query head);
//  * one thread streams the split's K/V tiles by TMA (no multicast) into a
//    shared ring of 64- or 128-key stages; each of the 4 warps takes its own
//    quarter of the keys of every stage, and a stage is refilled once all
//    four have left it; the first stages and the Q rows are prefetched into
//    L2 before the dependent-launch wait;
//  * QK^T and PV use warp-level m16n8k16 MMAs (ldmatrix operands) with an
//    online softmax in the exp2 domain; the 4 warps' (m, l, O) are merged in
//    shared memory at the end;
//  * with one split the CTA writes O/LSE directly, otherwise fp32 partials
//    (O normalised, LSE natural log) that the merge kernel combines.
#include <math.h>

#include <string.h>

#include <mutex>
#include <utility>

#include "kf_host.h"
#include "kf_sm100.cuh"

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct DecodeArgs {
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  const uint16_t* nk;  // fused-append source rows (null when not fused)
  const uint16_t* nv;
  uint16_t* kw;  // cache base for the fused append write
  uint16_t* vw;
  uint16_t* o;
  float* lse;
  float* part_o;
  float* part_lse;
  int64_t qs[4], ks[4], vs[4], nks[4], nvs[4], os[4];
  int B, Hq, Hkv, G, Sq, Sk, D;
  int64_t past_len;
  int num_splits, chunk;
  bool direct;  // one split writing O/LSE itself; otherwise fp32 partials for a merge
  int rows;  // G * Sq packed rows per KV head
  int64_t prow_total;  // B * Hq * Sq
  float scale_log2;
  int32_t* status;     // device word set when a bounded wait expires (may be null)
};

__device__ __forceinline__ uint32_t swz(int row, int chunk, int row_bytes) {
  return (uint32_t)(row * row_bytes + ((((chunk & 7) ^ (row & 7)) | (chunk & ~7)) << 4));
}

__device__ __forceinline__ float warp_max4(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
  return x;
}

// Shared-memory address of 16-byte chunk `c` of row `r` in a TMA tile stored
// as 64-column panels of `rows` x 128 B with the 128-byte swizzle.
__device__ __forceinline__ uint32_t tma_swz(int r, int c, int rows) {
  return (uint32_t)((c >> 3) * rows * 128 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Keys per K/V tile: 4 warps x 16 keys, or 4 x 32 on the transposed path for
// head_dim <= 64 (fewer, larger steps per warp).
__host__ __device__ constexpr int tile_keys(int kw) { return kWarps * kw; }

// NP = 64-column panels of the padded head dim (1 or 2), MT = 16-row m-tiles of
// packed query rows, STAGES = depth of the K/V ring.
//
// N8 (at most 8 packed rows, e.g. one query token of a 4-way GQA group): the
// products are taken transposed, S^T = K Q^T and O^T = V^T P^T, so the query
// rows sit on the MMA's n = 8 side instead of padding a 16-row m tile.  That
// halves the MMAs per key (the legacy warp MMA is what bounds this kernel at
// small row counts).  P^T goes from the S^T accumulator layout to the B
// operand layout with movmatrix (8x8 transposes in registers); the row max
// and sum reduce across the 8 lane groups that hold a row's keys.
template <bool BF16, int NP, int MT, int STAGES, bool N8, int KW>
__global__ void __launch_bounds__(kThreads)
decode_split_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                    const DecodeArgs a) {
  constexpr int DP = NP * 64;
  constexpr int ROWS = N8 ? 8 : MT * 16;
  constexpr int Q_ROW_BYTES = DP * 2;
  constexpr int CHUNKS = DP / 8;                 // 16-byte chunks per row
  constexpr int TN = tile_keys(KW);              // keys per K/V tile (KW per warp)
  constexpr int PANEL = TN * 128;                // one 64-column panel of a tile
  constexpr int TILE = NP * PANEL;               // K (or V) tile bytes
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sKV = smem;                           // [stage][K tile | V tile]
  uint8_t* sQ = smem + STAGES * 2 * TILE;        // [ROWS][DP] (row-local XOR swizzle)
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES];
  __shared__ int abort_any;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x;
  const int b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int row0 = blockIdx.z * ROWS;
  const int key_begin = split * a.chunk;
  const int key_end = min(key_begin + a.chunk, a.Sk);
  const int n_tiles = (key_end - key_begin + TN - 1) / TN;
  const bool fused = a.nk != nullptr;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      kf::mbar_init(&full[s], 1);
      kf::mbar_init(&empty[s], kWarps);
    }
    kf::fence_barrier_init();
    abort_any = 0;
    kf::tma_prefetch_desc(&map_k);
    kf::tma_prefetch_desc(&map_v);
    // the first tiles' HBM latency overlaps the previous kernel's tail (an
    // L2 prefetch only hints: L2 stays coherent with that kernel's writes)
    for (int t = 0; t < STAGES && t < n_tiles; ++t)
#pragma unroll
      for (int pn = 0; pn < NP; ++pn) {
        kf::tma_prefetch_l2_4d(&map_k, pn * 64, key_begin + t * TN, kvh, b);
        kf::tma_prefetch_l2_4d(&map_v, pn * 64, key_begin + t * TN, kvh, b);
      }
  }
  if (tid < ROWS && row0 + tid < a.rows) {
    const int pr = row0 + tid, g = pr / a.Sq, s = pr % a.Sq;
    kf::prefetch_l2_bulk(a.q + b * a.qs[0] + (int64_t)(kvh * a.G + g) * a.qs[1] + s * a.qs[2], a.D * 2);
  }
  // Launched with programmatic stream serialization: everything above ran
  // while the previous kernel of the stream may still be finishing; nothing
  // below may start before it has completed.  The merge kernel that follows
  // may be scheduled from here on (it waits for this grid the same way).
  kf::griddep_wait();
  kf::griddep_launch_dependents();
  __syncthreads();
  int issued = 0;  // tiles whose loads thread 0 has issued
  // one thread streams K/V tiles (TMA, no multicast); the ring is recycled
  // once all four warps have released a stage
  auto issue = [&](int t) {
    const int s = t % STAGES;
    uint8_t* kt = sKV + s * 2 * TILE;
    kf::mbar_arrive_expect_tx(&full[s], 2 * TILE);
#pragma unroll
    for (int pn = 0; pn < NP; ++pn) {
      kf::tma_load_4d(kt + pn * PANEL, &map_k, &full[s], pn * 64, key_begin + t * TN, kvh, b);
      kf::tma_load_4d(kt + TILE + pn * PANEL, &map_v, &full[s], pn * 64, key_begin + t * TN, kvh, b);
    }
  };
  if (tid == 0) {
    for (int t = 0; t < STAGES && t < n_tiles; ++t) issue(t);
    issued = min(STAGES, n_tiles);
  }

  // fused append: the CTA of the split owning the new position (row block 0)
  // writes the new K/V row into the cache; every CTA substitutes it in smem.
  if (fused && blockIdx.z == 0 && a.past_len >= key_begin && a.past_len < key_end && warp == 1) {
    for (int c = lane; c < a.D / 8; c += 32) {
      const uint4 kv = *reinterpret_cast<const uint4*>(a.nk + b * a.nks[0] + kvh * a.nks[1] + c * 8);
      const uint4 vv = *reinterpret_cast<const uint4*>(a.nv + b * a.nvs[0] + kvh * a.nvs[1] + c * 8);
      *reinterpret_cast<uint4*>(a.kw + b * a.ks[0] + kvh * a.ks[1] + a.past_len * a.ks[2] + c * 8) = kv;
      *reinterpret_cast<uint4*>(a.vw + b * a.vs[0] + kvh * a.vs[1] + a.past_len * a.vs[2] + c * 8) = vv;
    }
  }

  // ---- Q tile (packed rows), zero-filled outside [rows) x [D)
  for (int i = tid; i < ROWS * CHUNKS; i += kThreads) {
    const int r = i / CHUNKS, c = i % CHUNKS;
    const int pr = row0 + r;
    const bool ok = pr < a.rows && c * 8 < a.D;
    const int g = ok ? pr / a.Sq : 0, s = ok ? pr % a.Sq : 0;
    const uint16_t* src = a.q + b * a.qs[0] + (int64_t)(kvh * a.G + g) * a.qs[1] + s * a.qs[2] + (ok ? c * 8 : 0);
    kf::cp_async16(sQ + swz(r, c, Q_ROW_BYTES), src, ok);
  }
  kf::cp_async_commit();
  kf::cp_async_wait<0>();
  __syncthreads();

  float m_run[MT][2], l_run[MT][2];
  float o_acc[MT][DP / 8][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    m_run[mt][0] = m_run[mt][1] = -INFINITY;
    l_run[mt][0] = l_run[mt][1] = 0.f;
#pragma unroll
    for (int n = 0; n < DP / 8; ++n) o_acc[mt][n][0] = o_acc[mt][n][1] = o_acc[mt][n][2] = o_acc[mt][n][3] = 0.f;
  }
  const uint32_t sQ_u = kf::smem_u32(sQ);
  const int wr0 = warp * KW;   // this warp's KW rows (keys) of every tile
  // N8 state: Q^T as B fragments (k = head dim, n = row), running max / sum
  // of rows 2 (lane % 4) + {0, 1}, and O^T accumulators (m = head dim).
  uint32_t qb[DP / 16][2];
  float m8[2] = {-INFINITY, -INFINITY}, l8[2] = {0.f, 0.f};
  float ot[DP / 16][4];
  if constexpr (N8) {
#pragma unroll
    for (int kk = 0; kk < DP / 16; kk += 2) {
      uint32_t r4[4];
      kf::ldmatrix_x4(r4, sQ_u + swz(lane & 7, 2 * kk + (lane >> 3), Q_ROW_BYTES));
      qb[kk][0] = r4[0];
      qb[kk][1] = r4[1];
      qb[kk + 1][0] = r4[2];
      qb[kk + 1][1] = r4[3];
    }
#pragma unroll
    for (int dm = 0; dm < DP / 16; ++dm) ot[dm][0] = ot[dm][1] = ot[dm][2] = ot[dm][3] = 0.f;
  }
  bool ok = true;
  int t_stop = n_tiles;
  for (int t = 0; t < n_tiles; ++t) {
    const int st = t % STAGES;
    const uint32_t ph = (t / STAGES) & 1;
    // thread 0 refills the stage freed by the previous tile once all warps left it
    if (tid == 0 && t > 0 && t - 1 + STAGES < n_tiles) {
      const int sp = (t - 1) % STAGES;
      if (kf::mbar_wait(&empty[sp], ((t - 1) / STAGES) & 1, a.status)) {
        issue(t - 1 + STAGES);
        issued = t + STAGES;
      } else {
        abort_any = 1;
      }
    }
    // warp-uniform outcome: no lane reaches the collective ldmatrix/mma alone
    ok = __all_sync(0xffffffffu, kf::mbar_wait(&full[st], ph, a.status) && !*(volatile int*)&abort_any);
    if (!ok) {
      t_stop = t;
      if (lane == 0) abort_any = 1;
      break;
    }
    uint8_t* kt = sKV + st * 2 * TILE;
    uint8_t* vt = kt + TILE;
    const int key0 = key_begin + t * TN + wr0;
    if (fused && a.past_len >= key0 && a.past_len < key0 + KW) {
      const int r = wr0 + (int)(a.past_len - key0);
      for (int c = lane; c < CHUNKS; c += 32) {
        const bool in = c * 8 < a.D;
        const uint4 kv = in ? *reinterpret_cast<const uint4*>(a.nk + b * a.nks[0] + kvh * a.nks[1] + c * 8) : make_uint4(0, 0, 0, 0);
        const uint4 vv = in ? *reinterpret_cast<const uint4*>(a.nv + b * a.nvs[0] + kvh * a.nvs[1] + c * 8) : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(kt + tma_swz(r, c, TN)) = kv;
        *reinterpret_cast<uint4*>(vt + tma_swz(r, c, TN)) = vv;
      }
      __syncwarp();
    }
    const uint32_t sk_u = kf::smem_u32(kt), sv_u = kf::smem_u32(vt);

    if constexpr (N8) {
      // S^T (KW keys x 8 rows) = K Q^T, as KW / 16 independent 16-key halves
      constexpr int H = KW / 16;
      float c[H][4];
#pragma unroll
      for (int h = 0; h < H; ++h) c[h][0] = c[h][1] = c[h][2] = c[h][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk)
#pragma unroll
        for (int h = 0; h < H; ++h) {
          uint32_t ka[4];
          kf::ldmatrix_x4(ka, sk_u + tma_swz(wr0 + h * 16 + (lane & 15), 2 * kk + (lane >> 4), TN));
          kf::mma_16816<BF16>(c[h], ka, qb[kk][0], qb[kk][1]);
        }
      // rows 2 (lane % 4) + {0, 1}; keys h*16 + lane / 4 (c0, c1) and + 8 (c2, c3)
      float x[H][4];
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int h = 0; h < H; ++h) {
        const int ka0 = key0 + h * 16 + (lane >> 2);
        x[h][0] = ka0 < key_end ? c[h][0] * a.scale_log2 : -INFINITY;
        x[h][1] = ka0 < key_end ? c[h][1] * a.scale_log2 : -INFINITY;
        x[h][2] = ka0 + 8 < key_end ? c[h][2] * a.scale_log2 : -INFINITY;
        x[h][3] = ka0 + 8 < key_end ? c[h][3] * a.scale_log2 : -INFINITY;
        mx[0] = kf::fmax3(mx[0], x[h][0], x[h][2]);
        mx[1] = kf::fmax3(mx[1], x[h][1], x[h][3]);
      }
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], off));
        mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], off));
      }
      float alpha[2], mu[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float m_new = fmaxf(m8[j], mx[j]);
        mu[j] = m_new == -INFINITY ? 0.f : m_new;
        alpha[j] = kf::ex2(m8[j] - mu[j]);
        m8[j] = m_new;
      }
      float pp[H][4];
      float ls[2] = {0.f, 0.f};
#pragma unroll
      for (int h = 0; h < H; ++h) {
        pp[h][0] = kf::ex2(x[h][0] - mu[0]);
        pp[h][1] = kf::ex2(x[h][1] - mu[1]);
        pp[h][2] = kf::ex2(x[h][2] - mu[0]);
        pp[h][3] = kf::ex2(x[h][3] - mu[1]);
        ls[0] += pp[h][0] + pp[h][2];
        ls[1] += pp[h][1] + pp[h][3];
      }
      l8[0] = l8[0] * alpha[0] + ls[0];
      l8[1] = l8[1] * alpha[1] + ls[1];
      if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
        for (int dm = 0; dm < DP / 16; ++dm) {
          ot[dm][0] *= alpha[0];
          ot[dm][1] *= alpha[1];
          ot[dm][2] *= alpha[0];
          ot[dm][3] *= alpha[1];
        }
      }
      // P^T as the B operand (k = key, n = row): transpose the 8x8 blocks
      uint32_t pb[H][2];
#pragma unroll
      for (int h = 0; h < H; ++h) {
        pb[h][0] = kf::movmatrix_trans(kf::pack2<BF16>(pp[h][0], pp[h][1]));
        pb[h][1] = kf::movmatrix_trans(kf::pack2<BF16>(pp[h][2], pp[h][3]));
      }
      // O^T (head dim x 8 rows) += V^T P^T
#pragma unroll
      for (int dm = 0; dm < DP / 16; ++dm)
#pragma unroll
        for (int h = 0; h < H; ++h) {
          uint32_t va[4];
          kf::ldmatrix_x4_trans(va, sv_u + tma_swz(wr0 + h * 16 + (lane & 7) + ((lane >> 4) << 3),
                                                   2 * dm + ((lane >> 3) & 1), TN));
          kf::mma_16816<BF16>(ot[dm], va, pb[h][0], pb[h][1]);
        }
    } else {
      // S = Q K^T for this warp's 16 keys
      float sc[MT][2][4];
  #pragma unroll
      for (int mt = 0; mt < MT; ++mt)
  #pragma unroll
        for (int n = 0; n < 2; ++n) sc[mt][n][0] = sc[mt][n][1] = sc[mt][n][2] = sc[mt][n][3] = 0.f;
  #pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) {
        uint32_t kb[4];
        kf::ldmatrix_x4(kb, sk_u + tma_swz(wr0 + (lane & 7) + ((lane >> 4) << 3), 2 * kk + ((lane >> 3) & 1), TN));
  #pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          uint32_t qa[4];
          kf::ldmatrix_x4(qa, sQ_u + swz(mt * 16 + (lane & 15), 2 * kk + (lane >> 4), Q_ROW_BYTES));
          kf::mma_16816<BF16>(sc[mt][0], qa, kb[0], kb[1]);
          kf::mma_16816<BF16>(sc[mt][1], qa, kb[2], kb[3]);
        }
      }

      // online softmax (log2 domain), then O += P V
  #pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t pa[4];
  #pragma unroll
        for (int half = 0; half < 2; ++half) {
          float x[4];
  #pragma unroll
          for (int n = 0; n < 2; ++n)
  #pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int key = key0 + n * 8 + 2 * (lane & 3) + e;
              x[n * 2 + e] = key < key_end ? sc[mt][n][half * 2 + e] * a.scale_log2 : -INFINITY;
            }
          const float mx = warp_max4(fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])));
          const float m_new = fmaxf(m_run[mt][half], mx);
          const float m_use = m_new == -INFINITY ? 0.f : m_new;
          const float alpha = kf::ex2(m_run[mt][half] - m_use);
          float p[4];
  #pragma unroll
          for (int j = 0; j < 4; ++j) p[j] = kf::ex2(x[j] - m_use);
          l_run[mt][half] = l_run[mt][half] * alpha + (p[0] + p[1] + p[2] + p[3]);
          m_run[mt][half] = m_new;
          if (__any_sync(0xffffffffu, alpha != 1.f)) {  // skip when no row max moved
  #pragma unroll
            for (int n = 0; n < DP / 8; ++n) {
              o_acc[mt][n][half * 2 + 0] *= alpha;
              o_acc[mt][n][half * 2 + 1] *= alpha;
            }
          }
          pa[half] = kf::pack2<BF16>(p[0], p[1]);      // keys 0-7 of the warp's 16
          pa[2 + half] = kf::pack2<BF16>(p[2], p[3]);  // keys 8-15
        }
  #pragma unroll
        for (int dn = 0; dn < DP / 16; ++dn) {
          uint32_t vb[4];
          kf::ldmatrix_x4_trans(vb, sv_u + tma_swz(wr0 + (lane & 15), 2 * dn + (lane >> 4), TN));
          kf::mma_16816<BF16>(o_acc[mt][2 * dn], pa, vb[0], vb[1]);
          kf::mma_16816<BF16>(o_acc[mt][2 * dn + 1], pa, vb[2], vb[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) kf::mbar_arrive(&empty[st]);
  }

  // ---- merge the 4 warps in shared memory (reuses the ring: all tiles consumed)
  if constexpr (N8) {
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) l8[j] += __shfl_xor_sync(0xffffffffu, l8[j], off);
  } else {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float l = l_run[mt][half];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        l_run[mt][half] = l;
      }
  }
  __syncthreads();
  if (abort_any) {
    // a bounded wait expired: let the loads already in flight land (bounded),
    // then make the failure visible as NaN outputs instead of stale data
    if (tid == 0)
      for (int t2 = t_stop; t2 < issued; ++t2)
        kf::mbar_wait(&full[t2 % STAGES], (t2 / STAGES) & 1, nullptr, 100000000ull);
    const int valid = min(ROWS, a.rows - row0);
    const int64_t pbase = (int64_t)(b * a.Hkv + kvh) * a.rows + row0;
    for (int i = tid; i < valid * a.D; i += kThreads) {
      const int r = i / a.D, c = i % a.D, pr = row0 + r;
      if (a.direct) {
        a.o[b * a.os[0] + (int64_t)(kvh * a.G + pr / a.Sq) * a.os[1] + (pr % a.Sq) * a.os[2] + c] = 0x7fffu;
      } else {
        a.part_o[((int64_t)split * a.prow_total + pbase + r) * a.D + c] = __int_as_float(0x7fc00000);
        if (c == 0) a.part_lse[(int64_t)split * a.prow_total + pbase + r] = 0.f;
      }
    }
    return;
  }
  float* ml = reinterpret_cast<float*>(smem);          // [warp][ROWS][2]
  float* row_w = ml + kWarps * ROWS * 2;               // [warp][ROWS] weights
  float* row_lse = row_w + kWarps * ROWS;              // [ROWS]
  float* obuf = row_lse + ROWS;                        // [warp][ROWS][DP]
  if constexpr (N8) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int r = 2 * (lane & 3) + j;
      if (lane < 4) {
        ml[(warp * ROWS + r) * 2 + 0] = m8[j];
        ml[(warp * ROWS + r) * 2 + 1] = l8[j];
      }
#pragma unroll
      for (int dm = 0; dm < DP / 16; ++dm) {
        const int d = dm * 16 + (lane >> 2);
        obuf[(warp * ROWS + r) * DP + d] = ot[dm][j];
        obuf[(warp * ROWS + r) * DP + d + 8] = ot[dm][2 + j];
      }
    }
  } else {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int r = mt * 16 + (lane >> 2) + half * 8;
        if ((lane & 3) == 0) {
          ml[(warp * ROWS + r) * 2 + 0] = m_run[mt][half];
          ml[(warp * ROWS + r) * 2 + 1] = l_run[mt][half];
        }
#pragma unroll
        for (int n = 0; n < DP / 8; ++n) {
          const int c = n * 8 + 2 * (lane & 3);
          obuf[(warp * ROWS + r) * DP + c] = o_acc[mt][n][half * 2];
          obuf[(warp * ROWS + r) * DP + c + 1] = o_acc[mt][n][half * 2 + 1];
        }
      }
  }
  __syncthreads();
  if (tid < ROWS) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, ml[(w * ROWS + tid) * 2]);
    float L = 0.f, wt[kWarps];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = ml[(w * ROWS + tid) * 2];
      wt[w] = (M == -INFINITY) ? 0.f : kf::ex2(mw - M);
      L += wt[w] * ml[(w * ROWS + tid) * 2 + 1];
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) row_w[w * ROWS + tid] = wt[w] * inv;
    row_lse[tid] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
  }
  __syncthreads();

  const int64_t prow_base = (int64_t)(b * a.Hkv + kvh) * a.rows + row0;
  const int valid_rows = min(ROWS, a.rows - row0);
  for (int i = tid; i < valid_rows * (DP / 4); i += kThreads) {
    const int r = i / (DP / 4), c4 = (i % (DP / 4)) * 4;
    if (c4 >= a.D) continue;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float wt = row_w[w * ROWS + r];
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] += wt * obuf[(w * ROWS + r) * DP + c4 + e];
    }
    const int pr = row0 + r;
    if (a.direct) {
      const int g = pr / a.Sq, s = pr % a.Sq;
      uint16_t* dst = a.o + b * a.os[0] + (int64_t)(kvh * a.G + g) * a.os[1] + s * a.os[2] + c4;
      const uint32_t lo = kf::pack2<BF16>(acc[0], acc[1]), hi = kf::pack2<BF16>(acc[2], acc[3]);
      *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
    } else {
      float* dst = a.part_o + ((int64_t)split * a.prow_total + prow_base + r) * a.D + c4;
      *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
  }
  if (tid < valid_rows) {
    if (a.direct) {
      if (a.lse) a.lse[prow_base + tid] = row_lse[tid];
    } else {
      a.part_lse[(int64_t)split * a.prow_total + prow_base + tid] = row_lse[tid];
    }
  }
}

// K3 on the tensor cores, for more than 16 packed rows (e.g. 4-way GQA with
// Sq >= 5) and no fused append: with several 16-row m tiles the warp-MMA
// version is bound by its MMAs, which tcgen05 takes off the critical path
// (one M = 128 tile covers up to 128 rows).
// CTA = (split, batch, KV head, block of up to 128 packed rows); rows sit on
// TMEM lanes (M = 128, unused lanes are zero rows whose warps skip the
// softmax).  Per 64-key tile: S = Q K^T (SS) into one of two S buffers,
// softmax by one thread per row (lazy rescale, P written back over S as
// 16-bit), O += P V (TS).  With two S buffers the next tile's S is computed
// while the softmax works on this one (one buffer measured 58% of HBM at
// Sq = 16, Sk = 131072; two: 65%).  Warps 0-3 softmax + Q load, warp 4 TMEM
// allocation + MMA issue, warp 5 TMA producer.  TMEM: S0 [0, 64), S1
// [64, 128), O [128, 128 + D).
constexpr int kTcThreads = 192;
constexpr int kTcKeys = 64;    // keys per K/V tile and per S buffer
constexpr int kTcStages = 4;
constexpr float kTcRescale = 8.0f;  // log2 units, as in the prefill forward
#ifndef KF_DEC_POLY_PAIRS
#define KF_DEC_POLY_PAIRS 2
#endif
constexpr int kTcPolyPairs = KF_DEC_POLY_PAIRS;  // of every 8 exponential pairs

struct __align__(8) TcBarriers {
  uint64_t full[kTcStages], empty[kTcStages];
  uint64_t q_ready, s_full[2], p_full[2], pv_done, o_done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, TcBarriers* bars, int32_t* status) {
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

template <bool BF16, int NP, int KS>
__global__ void __launch_bounds__(kTcThreads, 2)
decode_tc_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                 const DecodeArgs a) {
  constexpr int PANEL = kTcKeys * 128;   // K/V: 64 columns x kTcKeys rows, 128-byte swizzle
  constexpr int TILE = NP * PANEL;
  constexpr int QPANEL = 128 * 128;      // Q: 64 columns x 128 rows
  constexpr int d_pad16 = KS * 16;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sK = smem;                          // [stage][NP][128 keys][64]
  uint8_t* sV = sK + kTcStages * TILE;
  uint8_t* sQ = sV + kTcStages * TILE;         // [NP][128 rows][64]
  TcBarriers* bars = reinterpret_cast<TcBarriers*>(sQ + NP * QPANEL);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x;
  const int b = blockIdx.y / a.Hkv, kvh = blockIdx.y % a.Hkv;
  const int row0 = blockIdx.z * 128;
  const int valid_rows = min(128, a.rows - row0);
  const int active_warps = (valid_rows + 31) / 32;   // softmax warps holding real rows
  const int key_begin = split * a.chunk;
  const int key_end = min(key_begin + a.chunk, a.Sk);
  const int n_tiles = (key_end - key_begin + kTcKeys - 1) / kTcKeys;

  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      kf::mbar_init(&bars->full[s], 1);
      kf::mbar_init(&bars->empty[s], 1);
    }
    kf::mbar_init(&bars->q_ready, 128);
    for (int i = 0; i < 2; ++i) {
      kf::mbar_init(&bars->s_full[i], 1);
      kf::mbar_init(&bars->p_full[i], 32 * active_warps);
    }
    kf::mbar_init(&bars->pv_done, 1);
    kf::mbar_init(&bars->o_done, 1);
    bars->abort_flag = 0;
    kf::fence_barrier_init();
  }
  if (warp == 4) {
    kf::tmem_alloc(&bars->tmem_base, 256);
    kf::tmem_relinquish();
  }
  if (warp == 5 && lane == 0) {
    kf::tma_prefetch_desc(&map_k);
    kf::tma_prefetch_desc(&map_v);
    // the first tiles' HBM latency overlaps the previous kernel's tail
    for (int t = 0; t < kTcStages && t < n_tiles; ++t)
      for (int pn = 0; pn < NP; ++pn) {
        kf::tma_prefetch_l2_4d(&map_k, pn * 64, key_begin + t * kTcKeys, kvh, b);
        kf::tma_prefetch_l2_4d(&map_v, pn * 64, key_begin + t * kTcKeys, kvh, b);
      }
  }
  if (tid < valid_rows) {
    const int pr = row0 + tid, g = pr / a.Sq, s = pr % a.Sq;
    kf::prefetch_l2_bulk(a.q + b * a.qs[0] + (int64_t)(kvh * a.G + g) * a.qs[1] + s * a.qs[2], a.D * 2);
  }
  kf::tc_fence_before();
  __syncthreads();
  kf::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // programmatic dependent launch: see decode_split_kernel
  kf::griddep_wait();
  kf::griddep_launch_dependents();

  if (warp == 5) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      for (int t = 0; t < n_tiles; ++t) {
        const int s = t % kTcStages;
        if (!tc_wait(&bars->empty[s], ((t / kTcStages) & 1) ^ 1, bars, a.status)) break;
        ++issued;
        kf::mbar_arrive_expect_tx(&bars->full[s], 2 * TILE);
        for (int pn = 0; pn < NP; ++pn) {
          kf::tma_load_4d(sK + s * TILE + pn * PANEL, &map_k, &bars->full[s], pn * 64,
                          key_begin + t * kTcKeys, kvh, b);
          kf::tma_load_4d(sV + s * TILE + pn * PANEL, &map_v, &bars->full[s], pn * 64,
                          key_begin + t * kTcKeys, kvh, b);
        }
      }
      if (*(volatile int*)&bars->abort_flag) {
        // let loads still in flight land (bounded) before the CTA exits
        for (int t2 = max(0, issued - kTcStages); t2 < issued; ++t2)
          kf::mbar_wait(&bars->full[t2 % kTcStages], (t2 / kTcStages) & 1, nullptr, 100000000ull);
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = kf::make_idesc_f16(BF16, 128, kTcKeys, 0, 0);
      const uint32_t idesc_pv = kf::make_idesc_f16(BF16, 128, d_pad16, 0, 1);
      const kf::SDesc dq = kf::make_sdesc_split(kf::smem_u32(sQ), 16, 1024);
      const kf::SDesc dk = kf::make_sdesc_split(kf::smem_u32(sK), 16, 1024);
      const kf::SDesc dv = kf::make_sdesc_split(kf::smem_u32(sV), PANEL, 1024);
      // S is double-buffered (S_t in columns 64 (t & 1)): S_{t+1} = Q K_{t+1}^T
      // is issued before O += P_t V_t, so the softmax of tile t+1 can start
      // as soon as it finishes tile t.  S_{t+1} overwrites P_{t-1}, which
      // PV_{t-1} (issued earlier by this thread) has read.
      auto issue_qk = [&](int t) {
        const uint32_t koff = (t % kTcStages) * TILE;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          const uint32_t qo = (kk >> 2) * QPANEL + (kk & 3) * 32, ko = (kk >> 2) * PANEL + (kk & 3) * 32;
          kf::umma_ss(tmem + (t & 1) * kTcKeys, kf::sdesc_at(dq, qo), kf::sdesc_at(dk, koff + ko), idesc_qk,
                      kk > 0);
        }
        kf::umma_commit(&bars->s_full[t & 1]);
      };
      bool ok = tc_wait(&bars->q_ready, 0, bars, a.status) &&
                tc_wait(&bars->full[0], 0, bars, a.status);
      if (ok) {
        kf::tc_fence_after();
        issue_qk(0);
      }
      for (int t = 0; ok && t < n_tiles; ++t) {
        const int s = t % kTcStages;
        if (t + 1 < n_tiles) {
          if (!(ok = tc_wait(&bars->full[(t + 1) % kTcStages], ((t + 1) / kTcStages) & 1, bars, a.status))) break;
          kf::tc_fence_after();
          issue_qk(t + 1);
        }
        if (!(ok = tc_wait(&bars->p_full[t & 1], (t >> 1) & 1, bars, a.status))) break;
        kf::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTcKeys / 16; ++kk)
          kf::umma_ts(tmem + 128, tmem + (t & 1) * kTcKeys + kk * 8, kf::sdesc_at(dv, s * TILE + kk * 2048),
                      idesc_pv, (t > 0 || kk > 0));
        kf::umma_commit(&bars->empty[s]);
        kf::umma_commit(&bars->pv_done);
      }
      kf::umma_commit(&bars->o_done);
    }
  } else {
    // ------------------------------------------------------------ Q load + softmax (thread = row)
    constexpr int CH = NP * 8;  // 16-byte chunks per row
    {
      const int r = tid;        // tile row == TMEM lane
      const int pr = row0 + r;
      const bool in = r < valid_rows;
      const int g = in ? pr / a.Sq : 0, sq = in ? pr % a.Sq : 0;
      const uint16_t* src = a.q + b * a.qs[0] + (int64_t)(kvh * a.G + g) * a.qs[1] + sq * a.qs[2];
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const bool ok = in && c * 8 < a.D;
        kf::cp_async16(sQ + (c >> 3) * QPANEL + r * 128 + (((c & 7) ^ (r & 7)) << 4), src + (ok ? c * 8 : 0), ok);
      }
      kf::cp_async_commit();
      kf::cp_async_wait<0>();
      kf::fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
      kf::mbar_arrive(&bars->q_ready);
    }
    const int r = tid;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    float m_ref = -INFINITY, l_sum = 0.f;
    bool ok = true;
    if (warp < active_warps) {
      for (int t = 0; ok && t < n_tiles; ++t) {
        if (!(ok = __all_sync(0xffffffffu, tc_wait(&bars->s_full[t & 1], (t >> 1) & 1, bars, a.status)))) break;
        kf::tc_fence_after();
        const uint32_t s_col = (t & 1) * kTcKeys;
        uint32_t sr[kTcKeys];
        kf::tmem_ld32(lane_base + s_col + 0, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        kf::tmem_ld32(lane_base + s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        kf::tmem_wait_ld();
        const int key0 = key_begin + t * kTcKeys;
        const int lim = key_end - key0;  // keys past the split's end are masked
        if (lim < kTcKeys) {
#pragma unroll
          for (int c = 0; c < kTcKeys; ++c)
            if (c >= lim) sr[c] = 0xFF800000u;
        }
        float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll
        for (int c = 0; c < kTcKeys; c += 8) {
          a0 = kf::fmax3(a0, __uint_as_float(sr[c + 0]), __uint_as_float(sr[c + 1]));
          a1 = kf::fmax3(a1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
          a2 = kf::fmax3(a2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
          a3 = kf::fmax3(a3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
        }
        const float mx = kf::fmax3(a0, a1, fmaxf(a2, a3)) * a.scale_log2;
        float alpha = 1.f;
        bool rescale_o = false;
        if (t == 0) {
          m_ref = mx;
        } else if (mx > m_ref + kTcRescale) {
          alpha = kf::ex2(m_ref - mx);
          m_ref = mx;
          rescale_o = true;
        }
        const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
        l_sum *= alpha;
        const uint64_t scl = kf::f2(a.scale_log2, a.scale_log2), negm = kf::f2(-m_use, -m_use);
        uint32_t pk[kTcKeys / 2];
        uint64_t acc[2] = {0ull, 0ull};
        if (lim < kTcKeys) {
          // masked tile (-inf entries): MUFU only
#pragma unroll
          for (int c = 0; c < kTcKeys / 2; ++c) {
            float x0, x1;
            kf::f2_split(kf::fma2(kf::f2(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])), scl, negm), x0, x1);
            const float p0 = kf::ex2(x0), p1 = kf::ex2(x1);
            acc[c & 1] = kf::add2(acc[c & 1], kf::f2(p0, p1));
            pk[c] = kf::pack2<BF16>(p0, p1);
          }
        } else {
          // full tile: kTcPolyPairs of every 8 pairs on the fp32-pipe
          // polynomial, the rest on MUFU (with one live softmax warp per SM
          // sub-partition the exponentials are MUFU-bound otherwise)
#pragma unroll
          for (int c = 0; c < kTcKeys / 2; ++c) {
            float x0, x1;
            kf::f2_split(kf::fma2(kf::f2(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])), scl, negm), x0, x1);
            const uint64_t pp = (c & 7) < kTcPolyPairs ? kf::exp2_poly2(x0, x1) : kf::f2(kf::ex2(x0), kf::ex2(x1));
            acc[c & 1] = kf::add2(acc[c & 1], pp);
            float p0, p1;
            kf::f2_split(pp, p0, p1);
            pk[c] = kf::pack2<BF16>(p0, p1);
          }
        }
        {
          float s0, s1;
          kf::f2_split(kf::add2(acc[0], acc[1]), s0, s1);
          l_sum += s0 + s1;
        }
        kf::tmem_st32(lane_base + s_col, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
        if (__any_sync(0xffffffffu, rescale_o)) {
          // O row *= alpha once PV_{t-1} has landed (S_t was issued before it)
          if (!(ok = __all_sync(0xffffffffu, tc_wait(&bars->pv_done, (t - 1) & 1, bars, a.status)))) break;
          kf::tc_fence_after();
          for (int c0 = 0; c0 < d_pad16; c0 += 16) {
            uint32_t orow[16];
            kf::tmem_ld16(lane_base + 128 + c0, orow);
            kf::tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) orow[c] = __float_as_uint(__uint_as_float(orow[c]) * alpha);
            kf::tmem_st16(lane_base + 128 + c0, orow);
          }
        }
        kf::tmem_wait_st();
        kf::tc_fence_before();
        kf::mbar_arrive(&bars->p_full[t & 1]);
      }
      // ---------------------------------------------------------- epilogue
      if (__all_sync(0xffffffffu, ok && tc_wait(&bars->o_done, 0, bars, a.status))) {
        kf::tc_fence_after();
        const float inv_l = l_sum > 0.f ? 1.f / l_sum : 0.f;
        const float row_lse = l_sum > 0.f ? (m_ref + log2f(l_sum)) * kLn2 : -INFINITY;
        const bool row_ok = r < valid_rows;
        const int pr = row0 + r;
        const int64_t prow = (int64_t)(b * a.Hkv + kvh) * a.rows + pr;
        // O in 64-column batches: up to four 16-column loads in flight per
        // wait (one TMEM round trip per batch, on the tail of every split)
#pragma unroll
        for (int c0 = 0; c0 < d_pad16; c0 += 64) {
          uint32_t ov[64];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            if (c0 + 16 * q4 < d_pad16) {
              kf::tmem_ld16(lane_base + 128 + c0 + 16 * q4, *reinterpret_cast<uint32_t(*)[16]>(&ov[16 * q4]));
            } else {
#pragma unroll
              for (int c = 0; c < 16; ++c) ov[16 * q4 + c] = 0u;
            }
          }
          kf::tmem_wait_ld();
          if (!row_ok) continue;
          if (a.direct) {
            uint16_t* dst = a.o + b * a.os[0] + (int64_t)(kvh * a.G + pr / a.Sq) * a.os[1] + (pr % a.Sq) * a.os[2];
#pragma unroll
            for (int c = 0; c < 64; c += 2)
              if (c0 + c < a.D)
                *reinterpret_cast<uint32_t*>(dst + c0 + c) =
                    kf::pack2<BF16>(__uint_as_float(ov[c]) * inv_l, __uint_as_float(ov[c + 1]) * inv_l);
          } else {
            float* dst = a.part_o + ((int64_t)split * a.prow_total + prow) * a.D;
#pragma unroll
            for (int c = 0; c < 64; c += 4)
              if (c0 + c < a.D)
                *reinterpret_cast<float4*>(dst + c0 + c) =
                    make_float4(__uint_as_float(ov[c]) * inv_l, __uint_as_float(ov[c + 1]) * inv_l,
                                __uint_as_float(ov[c + 2]) * inv_l, __uint_as_float(ov[c + 3]) * inv_l);
          }
        }
        if (row_ok) {
          if (a.direct) {
            if (a.lse) a.lse[prow] = row_lse;
          } else {
            a.part_lse[(int64_t)split * a.prow_total + prow] = row_lse;
          }
        }
      }
    }
    if (!ok) {
      // a bounded wait expired: NaN outputs instead of stale data
      const int pr = row0 + r;
      if (r < valid_rows) {
        const int64_t prow = (int64_t)(b * a.Hkv + kvh) * a.rows + pr;
        for (int c = 0; c < a.D; ++c) {
          if (a.direct)
            a.o[b * a.os[0] + (int64_t)(kvh * a.G + pr / a.Sq) * a.os[1] + (pr % a.Sq) * a.os[2] + c] = 0x7fffu;
          else
            a.part_o[((int64_t)split * a.prow_total + prow) * a.D + c] = __int_as_float(0x7fc00000);
        }
        if (!a.direct) a.part_lse[(int64_t)split * a.prow_total + prow] = 0.f;
      }
    }
  }

  kf::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    kf::tc_fence_after();
    kf::tmem_dealloc(tmem, 256);
  }
}

// K3b: merge of S split partials by their LSE weights.
struct MergeArgs {
  const float* part_o;
  const float* part_lse;
  int S;
  int64_t rows;
  int D;
  uint16_t* o;
  float* lse;
  int Hq, Sq;
  int64_t os0, os1, os2;
};

// One 256-thread block per output row, built to need one round trip to L2:
// every thread first issues the loads of its partial-O chunks (thread (c, g)
// owns 4 columns c of splits g, g + G, ... with G = 256 / (D/4)), then the
// block reduces the partial LSEs (max, then the sum of weights) while those
// loads are in flight, and finally accumulates and reduces the G groups
// through shared memory.
constexpr int kMergeThreads = 256;
constexpr int kMergeBatch = 8;  // partial loads in flight per thread

// The merged row goes to out(c4, o4, lse): thread c4 < D/4 holds columns
// [4 c4, 4 c4 + 4), normalised; every such thread also gets the row's LSE.
template <class Out>
__device__ __forceinline__ void merge_row_to(const MergeArgs& a, const int64_t row, Out&& out) {
  extern __shared__ float sm[];          // [S] weights, then [G][D] partial sums
  float* wts = sm;
  float* part = sm + ((a.S + 3) & ~3);
  __shared__ float red[kMergeThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tpr = a.D / 4;               // threads per split (one 4-column chunk each)
  const int groups = kMergeThreads / tpr;
  const int c = tid % tpr, g = tid / tpr;
  const float* src = a.part_o + row * a.D + c * 4;
  const int64_t sstride = a.rows * a.D;

  float4 pb[kMergeBatch];
#pragma unroll
  for (int u = 0; u < kMergeBatch; ++u) {
    const int s = g + u * groups;
    pb[u] = s < a.S ? *reinterpret_cast<const float4*>(src + (int64_t)s * sstride) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // partial LSEs: S <= 2 * kMergeThreads
  float ls[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int s = tid + u * kMergeThreads;
    ls[u] = s < a.S ? a.part_lse[(int64_t)s * a.rows + row] : -INFINITY;
  }
  float mx = fmaxf(ls[0], ls[1]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < kMergeThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  float den = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int s = tid + u * kMergeThreads;
    const float w = (mx == -INFINITY || ls[u] == -INFINITY) ? 0.f : kf::ex2((ls[u] - mx) * kLog2e);
    if (s < a.S) wts[s] = w;
    den += w;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
  __syncthreads();  // red[] reads done, wts[] written
  if (lane == 0) red[warp] = den;
  __syncthreads();
  den = 0.f;
#pragma unroll
  for (int w = 0; w < kMergeThreads / 32; ++w) den += red[w];
  const float inv = den > 0.f ? 1.f / den : 0.f;

  if (g < groups) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int u = 0; u < kMergeBatch; ++u) {
      const int s = g + u * groups;
      const float w = s < a.S ? wts[s] : 0.f;
      acc[0] += w * pb[u].x;
      acc[1] += w * pb[u].y;
      acc[2] += w * pb[u].z;
      acc[3] += w * pb[u].w;
    }
    for (int s0 = g + kMergeBatch * groups; s0 < a.S; s0 += kMergeBatch * groups) {
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) {
        const int s = s0 + u * groups;
        pb[u] = s < a.S ? *reinterpret_cast<const float4*>(src + (int64_t)s * sstride) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) {
        const int s = s0 + u * groups;
        const float w = s < a.S ? wts[s] : 0.f;
        acc[0] += w * pb[u].x;
        acc[1] += w * pb[u].y;
        acc[2] += w * pb[u].z;
        acc[3] += w * pb[u].w;
      }
    }
    *reinterpret_cast<float4*>(part + g * a.D + c * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
  __syncthreads();
  if (tid < tpr) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int gg = 0; gg < groups; ++gg) {
      const float4 p = *reinterpret_cast<const float4*>(part + gg * a.D + tid * 4);
      acc[0] += p.x;
      acc[1] += p.y;
      acc[2] += p.z;
      acc[3] += p.w;
    }
    out(tid, make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv),
        den > 0.f ? mx + logf(den) : -INFINITY);
  }
}

// Output row `row` of a.o (strided [B, Hq, Sq, D]) and a.lse.
template <bool BF16>
__device__ __forceinline__ void merge_row(const MergeArgs& a, const int64_t row) {
  merge_row_to(a, row, [&](int c4, float4 v, float l) {
    const int64_t bh = row / a.Sq;
    const int64_t s_ = row % a.Sq;
    const int64_t b_ = bh / a.Hq, h_ = bh % a.Hq;
    uint16_t* dst = a.o + b_ * a.os0 + h_ * a.os1 + s_ * a.os2 + c4 * 4;
    *reinterpret_cast<uint2*>(dst) = make_uint2(kf::pack2<BF16>(v.x, v.y), kf::pack2<BF16>(v.z, v.w));
    if (c4 == 0 && a.lse) a.lse[row] = l;
  });
}

template <bool BF16>
__global__ void __launch_bounds__(kMergeThreads) merge_kernel(const MergeArgs a) {
  kf::griddep_wait();  // partials of the split kernel (launched as its programmatic dependent)
  // The next decode call's split kernel may now be scheduled: its set-up
  // (barriers, TMEM, tensor maps) overlaps this merge, and it waits for the
  // merge to finish before it touches memory (0.3-0.7 us per call).
  kf::griddep_launch_dependents();
  merge_row<BF16>(a, blockIdx.x);
}

// Launch with programmatic stream serialization: the kernel may be scheduled
// before the previous kernel in the stream finishes and orders itself with
// griddepcontrol.wait, hiding launch latency between back-to-back kernels
// (split -> merge, and one decode step -> the next).
template <typename... KArgs, typename... Args>
int launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) != cudaSuccess) {
    (void)cudaGetLastError();
    return kf::set_error(KF_ERR_CUDA, "%s: launch failed", what);
  }
  return kf::check_launch(what);
}

// Keys per K/V tile of the kernel variant dispatch_split picks; split chunks
// are multiples of it.
int decode_tile_keys(int64_t rows, int64_t D, bool fused) {
  if (rows > 16 && !fused) return kTcKeys;
  return (rows <= 8 && D <= 64) ? tile_keys(32) : tile_keys(16);
}

template <bool BF16>
int launch_merge(const MergeArgs& m, cudaStream_t st) {
  const int groups = kMergeThreads / (m.D / 4);
  const size_t smem = (size_t)(((m.S + 3) & ~3) + groups * m.D) * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(merge_kernel<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return kf::set_error(KF_ERR_CUDA, "kf merge: cannot reserve %zu bytes of shared memory", smem);
  if (m.rows > 0x7fffffffLL) return kf::set_error(KF_ERR_UNSUPPORTED, "kf merge: too many rows");
  return launch_dependent(merge_kernel<BF16>, dim3((unsigned)m.rows), dim3(kMergeThreads), smem, st, "kf merge", m);
}

template <bool BF16, int NP, int MT, bool N8 = false, int KW = 16>
int launch_split(const DecodeArgs& a, const CUtensorMap& mk, const CUtensorMap& mv, int row_blocks,
                 cudaStream_t st) {
  constexpr int STAGES = KW == 32 ? 3 : (NP == 1 ? 4 : 2);
  constexpr int DP = NP * 64;
  constexpr int ROWS = N8 ? 8 : MT * 16;
  const size_t pipe = 1024 + (size_t)STAGES * 2 * NP * tile_keys(KW) * 128 + (size_t)ROWS * DP * 2;
  const size_t merge = 1024 + (size_t)kWarps * ROWS * 3 * 4 + ROWS * 4 + (size_t)kWarps * ROWS * DP * 4;
  const size_t smem = pipe > merge ? pipe : merge;
  auto kern = decode_split_kernel<BF16, NP, MT, STAGES, N8, KW>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return kf::set_error(KF_ERR_CUDA, "kf_decode: cannot reserve %zu bytes of shared memory", smem);
  dim3 grid(a.num_splits, a.B * a.Hkv, row_blocks);
  return launch_dependent(kern, grid, dim3(kThreads), smem, st, "kf_decode", mk, mv, a);
}

template <bool BF16, int KS>
int launch_tc(const DecodeArgs& a, const CUtensorMap& mk, const CUtensorMap& mv, cudaStream_t st) {
  constexpr int NP = KS > 4 ? 2 : 1;
  constexpr size_t TILE = (size_t)NP * kTcKeys * 128;
  const size_t smem = 1024 + 2 * kTcStages * TILE + (size_t)NP * 128 * 128 + sizeof(TcBarriers);
  auto kern = decode_tc_kernel<BF16, NP, KS>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return kf::set_error(KF_ERR_CUDA, "kf_decode: cannot reserve %zu bytes of shared memory", smem);
  dim3 grid(a.num_splits, a.B * a.Hkv, (a.rows + 127) / 128);
  return launch_dependent(kern, grid, dim3(kTcThreads), smem, st, "kf_decode", mk, mv, a);
}

template <bool BF16>
int dispatch_tc(const DecodeArgs& a, const kf_tensor4* k, const kf_tensor4* v, cudaStream_t st) {
  CUtensorMap mk, mv;
  int rc;
  if ((rc = kf::encode_tmap_4d(&mk, k, 64, kTcKeys))) return rc;
  if ((rc = kf::encode_tmap_4d(&mv, v, 64, kTcKeys))) return rc;
  switch ((a.D + 15) / 16) {
    case 1: return launch_tc<BF16, 1>(a, mk, mv, st);
    case 2: return launch_tc<BF16, 2>(a, mk, mv, st);
    case 3: return launch_tc<BF16, 3>(a, mk, mv, st);
    case 4: return launch_tc<BF16, 4>(a, mk, mv, st);
    case 5: return launch_tc<BF16, 5>(a, mk, mv, st);
    case 6: return launch_tc<BF16, 6>(a, mk, mv, st);
    case 7: return launch_tc<BF16, 7>(a, mk, mv, st);
    default: return launch_tc<BF16, 8>(a, mk, mv, st);
  }
}

template <bool BF16>
int dispatch_split(const DecodeArgs& a, const kf_tensor4* k, const kf_tensor4* v, cudaStream_t st) {
  if (a.rows > 16 && a.nk == nullptr) return dispatch_tc<BF16>(a, k, v, st);
  CUtensorMap mk, mv;
  int rc;
  const int np = a.D <= 64 ? 1 : 2;
  const int tn = decode_tile_keys(a.rows, a.D, a.nk != nullptr);
  if ((rc = kf::encode_tmap_4d(&mk, k, 64, tn))) return rc;
  if ((rc = kf::encode_tmap_4d(&mv, v, 64, tn))) return rc;
  if (a.rows <= 8)  // transposed products: rows on the n = 8 side
    return np == 1 ? launch_split<BF16, 1, 1, true, 32>(a, mk, mv, 1, st)
                   : launch_split<BF16, 2, 1, true, 16>(a, mk, mv, 1, st);
  const int mt_max = np == 1 ? 4 : 2;
  int mt = (a.rows + 15) / 16;
  if (mt > mt_max) mt = mt_max;
  const int row_blocks = (a.rows + mt * 16 - 1) / (mt * 16);
  if (np == 1) {
    switch (mt) {
      case 1: return launch_split<BF16, 1, 1>(a, mk, mv, row_blocks, st);
      case 2: return launch_split<BF16, 1, 2>(a, mk, mv, row_blocks, st);
      case 3: return launch_split<BF16, 1, 3>(a, mk, mv, row_blocks, st);
      default: return launch_split<BF16, 1, 4>(a, mk, mv, row_blocks, st);
    }
  }
  if (mt == 1) return launch_split<BF16, 2, 1>(a, mk, mv, row_blocks, st);
  return launch_split<BF16, 2, 2>(a, mk, mv, row_blocks, st);
}

bool rows16(const kf_tensor4* t) {
  if (!t || !kf::aligned16(t->ptr) || t->stride[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (t->size[i] > 1 && (t->stride[i] % 8) != 0) return false;
  return true;
}

int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace

// Mirrors kotflash_b200/_planning.py:split_kv_plan (same formula).
extern "C" int kf_decode_num_splits(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk,
                                    int64_t D, int sm_count) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Sk <= 0 || D <= 0) return 1;
  if (sm_count <= 0) sm_count = 148;
  const int64_t group = Hq / Hkv > 0 ? Hq / Hkv : 1;
  const int64_t rows_per_cta = D <= 64 ? 64 : 32;
  const int64_t units = B * Hkv * cdiv64(group * Sq, rows_per_cta);
  // at least one 64-key tile per split: below ~16K keys a split's time is its
  // pipeline latency, so more, shorter splits finish sooner (cfg3, Sq=1:
  // Sk=1024 6.4 -> 5.8 us; Sq=4: 7.9 -> 6.2 us)
  const int64_t max_by_len = cdiv64(Sk, 64) > 1 ? cdiv64(Sk, 64) : 1;
  int64_t splits = cdiv64(2 * (int64_t)sm_count, units);
  if (splits > max_by_len) splits = max_by_len;
  if (splits > 512) splits = 512;
  if (splits < 1) splits = 1;
  const int64_t chunk = cdiv64(cdiv64(Sk, splits), 64) * 64;
  return (int)cdiv64(Sk, chunk);
}

extern "C" size_t kf_decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Sq, int64_t D,
                                            int num_splits) {
  if (num_splits <= 1) return 0;
  return (size_t)num_splits * (size_t)(B * Hq * Sq) * (size_t)(D + 1) * sizeof(float) + 256;
}

namespace {

// Validates the descriptors and fills `a`: split geometry and, when the
// splits write fp32 partials (more than one split, or `partials` forced), the
// workspace carve-up.  Messages are prefixed with `what`.
int decode_setup(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v, const kf_tensor4* new_k,
                 const kf_tensor4* new_v, int64_t past_len, const kf_tensor4* o, float* lse, int dtype,
                 float scale, int num_splits, void* workspace, size_t workspace_bytes, bool partials,
                 const char* what, DecodeArgs& a) {
  using kf::set_error;
  if (!q || !k || !v || !o) return set_error(KF_ERR_INVALID, "%s: null tensor descriptor", what);
  if (dtype != KF_F16 && dtype != KF_BF16)
    return set_error(KF_ERR_INVALID, "%s: dtype must be fp16 or bf16", what);
  const int64_t B = q->size[0], Hq = q->size[1], Sq = q->size[2], D = q->size[3];
  const int64_t Hkv = k->size[1], Sk = k->size[2];
  for (int i = 0; i < 4; ++i)
    if (k->size[i] != v->size[i]) return set_error(KF_ERR_INVALID, "%s: K and V shapes must match", what);
  if (k->size[0] != B || k->size[3] != D)
    return set_error(KF_ERR_INVALID, "%s: K/V batch and head_dim must match Q", what);
  for (int i = 0; i < 4; ++i)
    if (o->size[i] != q->size[i]) return set_error(KF_ERR_INVALID, "%s: O must have Q's shape", what);
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Sk <= 0)
    return set_error(KF_ERR_INVALID, "%s: dimensions must be non-zero", what);
  if (Hq % Hkv != 0)
    return set_error(KF_ERR_INVALID, "%s: num_query_heads must be divisible by num_kv_heads", what);
  if (Sq > 16) return set_error(KF_ERR_UNSUPPORTED, "%s: Sq must be <= 16", what);
  if (D < 16 || D > 128 || D % 8 != 0)
    return set_error(KF_ERR_UNSUPPORTED, "%s: head_dim must be a multiple of 8 in [16, 128]", what);
  if (Sk > (int64_t)1 << 30) return set_error(KF_ERR_UNSUPPORTED, "%s: Sk too large", what);
  if (!rows16(q) || !rows16(k) || !rows16(v) || !rows16(o))
    return set_error(KF_ERR_INVALID, "%s: tensors need a contiguous last dim and 16-byte aligned rows", what);
  const bool fused = new_k != nullptr || new_v != nullptr;
  if (fused) {
    if (!new_k || !new_v) return set_error(KF_ERR_INVALID, "%s: new_k and new_v go together", what);
    if (new_k->size[0] != B || new_k->size[1] != Hkv || new_k->size[2] != 1 || new_k->size[3] != D)
      return set_error(KF_ERR_INVALID, "%s: new K/V must be [B, Hkv, 1, D]", what);
    for (int i = 0; i < 4; ++i)
      if (new_v->size[i] != new_k->size[i])
        return set_error(KF_ERR_INVALID, "%s: new K and V shapes must match", what);
    if (!rows16(new_k) || !rows16(new_v))
      return set_error(KF_ERR_INVALID, "%s: new K/V rows must be 16-byte aligned", what);
    if (past_len != Sk - 1)
      return set_error(KF_ERR_INVALID, "%s: fused append needs past_len == Sk - 1", what);
  }
  if (num_splits <= 0)
    num_splits = kf_decode_num_splits(B, Hq, Hkv, Sq, Sk, D, kf::sm_count_current_device());
  if (num_splits > 65535) return set_error(KF_ERR_UNSUPPORTED, "%s: too many splits", what);
  const int64_t tk = decode_tile_keys(Hq / Hkv * Sq, D, fused);
  const int64_t chunk = cdiv64(cdiv64(Sk, num_splits), tk) * tk;
  num_splits = (int)cdiv64(Sk, chunk);

  a = DecodeArgs{};
  a.q = static_cast<const uint16_t*>(q->ptr);
  a.k = static_cast<const uint16_t*>(k->ptr);
  a.v = static_cast<const uint16_t*>(v->ptr);
  a.nk = fused ? static_cast<const uint16_t*>(new_k->ptr) : nullptr;
  a.nv = fused ? static_cast<const uint16_t*>(new_v->ptr) : nullptr;
  a.kw = static_cast<uint16_t*>(k->ptr);
  a.vw = static_cast<uint16_t*>(v->ptr);
  a.o = static_cast<uint16_t*>(o->ptr);
  a.lse = lse;
  for (int i = 0; i < 4; ++i) {
    a.qs[i] = q->stride[i];
    a.ks[i] = k->stride[i];
    a.vs[i] = v->stride[i];
    a.os[i] = o->stride[i];
    a.nks[i] = fused ? new_k->stride[i] : 0;
    a.nvs[i] = fused ? new_v->stride[i] : 0;
  }
  a.B = (int)B;
  a.Hq = (int)Hq;
  a.Hkv = (int)Hkv;
  a.G = (int)(Hq / Hkv);
  a.Sq = (int)Sq;
  a.Sk = (int)Sk;
  a.D = (int)D;
  a.past_len = past_len;
  a.num_splits = num_splits;
  a.chunk = (int)chunk;
  a.rows = a.G * a.Sq;
  a.prow_total = B * Hq * Sq;
  a.scale_log2 = scale * kLog2e;
  a.part_o = nullptr;
  a.part_lse = nullptr;
  a.status = nullptr;
  a.direct = num_splits == 1 && !partials;
  if (!a.direct) {
    const size_t need = (size_t)num_splits * (size_t)(B * Hq * Sq) * (size_t)(D + 1) * sizeof(float) + 256;
    if (!workspace || workspace_bytes < need)
      return set_error(KF_ERR_WORKSPACE, "%s: workspace needs %zu bytes", what, need);
    uintptr_t base = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255);
    a.part_o = reinterpret_cast<float*>(base);
    a.part_lse = a.part_o + (size_t)num_splits * a.prow_total * D;
  }
  if (a.G * a.Sq > (1 << 20)) return set_error(KF_ERR_UNSUPPORTED, "%s: too many rows per KV head", what);
  if ((int64_t)B * Hkv > 65535) return set_error(KF_ERR_UNSUPPORTED, "%s: B*Hkv too large", what);
  return KF_OK;
}

MergeArgs merge_args_of(const DecodeArgs& a) {
  MergeArgs m;
  m.part_o = a.part_o;
  m.part_lse = a.part_lse;
  m.S = a.num_splits;
  m.rows = a.prow_total;
  m.D = a.D;
  m.o = a.o;
  m.lse = a.lse;
  m.Hq = a.Hq;
  m.Sq = a.Sq;
  m.os0 = a.os[0];
  m.os1 = a.os[1];
  m.os2 = a.os[2];
  return m;
}

}  // namespace

extern "C" int kf_decode(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                         const kf_tensor4* new_k, const kf_tensor4* new_v, int64_t past_len,
                         const kf_tensor4* o, float* lse, int dtype, float scale, int num_splits,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!q) return kf::set_error(KF_ERR_INVALID, "kf_decode: null tensor descriptor");
  kf::DeviceGuard guard(q->ptr);
  if (guard.status()) return guard.status();
  DecodeArgs a;
  int rc = decode_setup(q, k, v, new_k, new_v, past_len, o, lse, dtype, scale, num_splits, workspace,
                        workspace_bytes, false, "kf_decode", a);
  if (rc != KF_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = dtype == KF_BF16 ? dispatch_split<true>(a, k, v, st) : dispatch_split<false>(a, k, v, st);
  if (rc != KF_OK || a.direct) return rc;
  const MergeArgs m = merge_args_of(a);
  return dtype == KF_BF16 ? launch_merge<true>(m, st) : launch_merge<false>(m, st);
}

extern "C" int kf_merge_partials(const float* part_o, const float* part_lse, int num_splits,
                                 int64_t rows, int64_t D, void* o, float* lse, int dtype,
                                 void* stream) {
  using kf::set_error;
  if (!part_o || !part_lse || !o) return set_error(KF_ERR_INVALID, "kf_merge_partials: null pointer");
  if (num_splits <= 0 || rows <= 0 || D <= 0 || D > 128 || D % 4 != 0)
    return set_error(KF_ERR_INVALID, "kf_merge_partials: need splits > 0, rows > 0, D % 4 == 0, D <= 128");
  if (num_splits > 2 * kMergeThreads)
    return set_error(KF_ERR_UNSUPPORTED, "kf_merge_partials: at most %d splits", 2 * kMergeThreads);
  if (dtype != KF_F16 && dtype != KF_BF16)
    return set_error(KF_ERR_INVALID, "kf_merge_partials: dtype must be fp16 or bf16");
  if ((reinterpret_cast<uintptr_t>(part_o) & 15) || (reinterpret_cast<uintptr_t>(o) & 7))
    return set_error(KF_ERR_INVALID, "kf_merge_partials: misaligned buffers");
  kf::DeviceGuard guard(part_o);
  if (guard.status()) return guard.status();
  MergeArgs m;
  m.part_o = part_o;
  m.part_lse = part_lse;
  m.S = num_splits;
  m.rows = rows;
  m.D = (int)D;
  m.o = static_cast<uint16_t*>(o);
  m.lse = lse;
  m.Hq = 1;
  m.Sq = 1;
  m.os0 = D;
  m.os1 = 0;
  m.os2 = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == KF_BF16 ? launch_merge<true>(m, st) : launch_merge<false>(m, st);
}

// ---------------------------------------------------------------------------
// Decode entry point that allocates nothing.
//
// Some callers cannot hand this library a workspace or let it allocate: a host
// runtime that owns every device allocation itself (an inference server's
// memory manager, or a JNI/cgo/ctypes embedder with a fixed device-memory
// budget) and gives plugins no allocator to call.  For them the split partials
// live in one file-scope device array of kNoAllocScratchBytes.  Every GPU that
// loads this library holds that array until the process exits.
//
// Set-up: every call, with the tensors' device current (the entry point makes
// it so), asks the runtime for the array's device address on that device
// (cudaGetSymbolAddress, a host-side lookup); nothing is cached, so the address
// stays right if the device's primary context is torn down and recreated.  The
// first call on a device also loads the module there, so make that first call
// before any stream capture.  Host code must never pass the array's name to a
// kernel: on the host it is only a stand-in.
//
// Sharing: all calls use the same array and it keeps the last call's
// contents.  Nothing needs clearing (every split writes each of its partial
// rows before the merge reads them), but calls that overlap on the GPU (two
// streams, or two threads' streams) race on the array: serialise them.
// ---------------------------------------------------------------------------

namespace {
constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB
__device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

int noalloc_scratch(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e != cudaSuccess || !p) {
    (void)cudaGetLastError();
    return kf::set_error(KF_ERR_CUDA, "kf_decode_noalloc: cudaGetSymbolAddress failed: %s",
                         cudaGetErrorString(e));
  }
  *out = p;
  return KF_OK;
}

int64_t effective_splits(int64_t Sk, int64_t s) {
  const int64_t chunk = cdiv64(cdiv64(Sk, s), 64) * 64;
  return cdiv64(Sk, chunk);
}
}  // namespace

extern "C" int kf_decode_noalloc(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                                 const kf_tensor4* new_k, const kf_tensor4* new_v,
                                 int64_t past_len, const kf_tensor4* o, float* lse, int dtype,
                                 float scale, int num_splits, void* stream) {
  if (!q || !k) return kf::set_error(KF_ERR_INVALID, "kf_decode_noalloc: null tensor descriptor");
  const int64_t B = q->size[0], Hq = q->size[1], Sq = q->size[2], D = q->size[3];
  const int64_t Hkv = k->size[1], Sk = k->size[2];
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Sk <= 0 || D <= 0)
    return kf::set_error(KF_ERR_INVALID, "kf_decode_noalloc: dimensions must be non-zero");
  kf::DeviceGuard guard(q->ptr);
  if (guard.status()) return guard.status();

  const size_t per_split = (size_t)(B * Hq * Sq) * (size_t)(D + 1) * sizeof(float);
  int64_t splits;
  if (num_splits > 0) {
    splits = effective_splits(Sk, num_splits);
    if (splits > 1 && kf_decode_workspace_bytes(B, Hq, Sq, D, (int)splits) > kNoAllocScratchBytes)
      return kf::set_error(KF_ERR_WORKSPACE,
                           "kf_decode_noalloc: %lld splits need %zu bytes of scratch, more than "
                           "the %zu-byte static maximum; pass fewer splits or use kf_decode",
                           (long long)splits,
                           kf_decode_workspace_bytes(B, Hq, Sq, D, (int)splits),
                           kNoAllocScratchBytes);
  } else {
    splits = effective_splits(
        Sk, kf_decode_num_splits(B, Hq, Hkv, Sq, Sk, D, kf::sm_count_current_device()));
    const int64_t fit = (int64_t)((kNoAllocScratchBytes - 256) / per_split);
    if (splits > fit) splits = fit >= 2 ? effective_splits(Sk, fit) : 1;
  }
  void* scratch = nullptr;
  if (splits > 1) {
    const int rc = noalloc_scratch(&scratch);
    if (rc != KF_OK) return rc;
  }
  return kf_decode(q, k, v, new_k, new_v, past_len, o, lse, dtype, scale, (int)splits, scratch,
                   splits > 1 ? kNoAllocScratchBytes : 0, stream);
}

// ---------------------------------------------------------------------------
// Cross-GPU exchange of decode partials through NVLink peer memory.
//
// Long-context decode splits the KV sequence over the ranks of one box; each
// rank ends with a partial (O, LSE) of its chunk, and every rank needs the
// merge of all of them.  Instead of a library all-gather followed by a merge
// launch, each rank owns a mailbox in its own memory that every peer can
// write (CUDA IPC mapping, peer access over NVLink/NVSwitch; no multicast):
//   put:   this rank's partial rows are stored (fp32) into slot [rank] of
//          every rank's mailbox with plain peer stores; then the sender adds
//          the row count to the receiver's arrival counter with release
//          semantics at system scope (a release reduction per piece in
//          kf_decode_peer_put; a system fence plus a relaxed reduction per
//          receiver, from parallel lanes, in the fused kv-split entry);
//   merge: every CTA waits (bounded) until its mailbox's counter shows all
//          W x rows rows of this call, then merges the W partials (the
//          split-merge math).
// Two producers exist: kf_decode_peer_put sends a finished (O, LSE), and the
// fused kv-split entry sends straight from the local merge of its splits
// (one kernel less, and no rounding of the partial to fp16/bf16).
//
// The call count (epoch) lives in the mailbox and is advanced by the last
// merge CTA, so the exchange works unchanged inside CUDA graphs.  Mailbox
// halves alternate by epoch parity; a rank cannot write epoch e + 2 into a
// half before every peer has finished merging epoch e from it (its merge of
// e + 1 needs their rows of e + 1, sent after their merge of e in stream
// order; with programmatic dependent launch every kernel of the next call
// still waits for the previous grid to complete before its first access).
// Counters only grow: after epoch e the counter of half (e & 1) holds
// W * rows * ((e + 1) / 2) modulo 2^32, and no intermediate value of an
// epoch equals it.
//
// Mailbox layout: [0, 256) control words {completed epochs, merge ticket,
// send ticket}, then two halves of {O [W][rows][D] fp32, LSE [W][rows] fp32,
// counter}.
namespace {

constexpr int kMaxPeers = 8;
constexpr int kPeerChunks = 16;
constexpr int kPeerThreads = 256;

struct PeerLayout {
  int64_t o_bytes, lse_bytes, half;
};

__host__ __device__ inline PeerLayout peer_layout(int world, int64_t rows, int D) {
  PeerLayout L;
  L.o_bytes = ((int64_t)world * rows * D * 4 + 255) & ~int64_t(255);
  L.lse_bytes = ((int64_t)world * rows * 4 + 255) & ~int64_t(255);
  L.half = L.o_bytes + L.lse_bytes + 256;
  return L;
}

// Rows per piece of kf_decode_peer_put (~16 KB of fp32 O per CTA, at most kPeerChunks pieces).
inline int64_t put_rows_per_piece(int64_t rows, int D) {
  int64_t pieces = (rows * D * 4 + 16383) / 16384;
  pieces = pieces < 1 ? 1 : (pieces > kPeerChunks ? kPeerChunks : pieces);
  return (rows + pieces - 1) / pieces;
}

struct PeerSet {
  uint8_t* mailbox[kMaxPeers];  // every rank's mailbox base, this rank's own included
};

struct PeerHalf {
  float* o;
  float* lse;
  uint32_t* counter;
};

KF_DEVI PeerHalf peer_half(uint8_t* mailbox, const PeerLayout& L, uint32_t e) {
  uint8_t* h = mailbox + 256 + (e & 1) * L.half;
  return {reinterpret_cast<float*>(h), reinterpret_cast<float*>(h + L.o_bytes),
          reinterpret_cast<uint32_t*>(h + L.o_bytes + L.lse_bytes)};
}

KF_DEVI uint32_t current_epoch(const uint8_t* mailbox) {
  return *reinterpret_cast<const volatile uint32_t*>(mailbox) + 1;
}

KF_DEVI void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
KF_DEVI void red_relaxed_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
KF_DEVI uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// grid (pieces, world): CTA (c, p) sends rows [c * rpp, (c + 1) * rpp) of this rank's partial to rank p.
template <bool BF16>
__global__ void __launch_bounds__(kPeerThreads) peer_put_kernel(const uint16_t* o, const float* lse, int64_t rows,
                                                                int D, int64_t rpp,
                                                                const __grid_constant__ PeerSet peers, int world,
                                                                int rank) {
  const PeerLayout L = peer_layout(world, rows, D);
  // The epoch is read before this CTA lets the merge launch: the merge's last
  // CTA advances it, and a dependent grid starts only once every CTA here has
  // triggered, so no CTA of this grid can see the next call's epoch.
  const uint32_t e = current_epoch(peers.mailbox[rank]);
  kf::griddep_launch_dependents();  // the merge waits for the counter, not for this grid
  const PeerHalf h = peer_half(peers.mailbox[blockIdx.y], L, e);
  const int64_t r0 = blockIdx.x * rpp, r1 = r0 + rpp < rows ? r0 + rpp : rows;
  if (r0 >= r1) return;
  float* dst_o = h.o + (int64_t)rank * rows * D;
  const int64_t per_row = D / 8;  // D % 8 == 0
  for (int64_t i = r0 * per_row + threadIdx.x; i < r1 * per_row; i += blockDim.x) {
    const uint4 v = reinterpret_cast<const uint4*>(o)[i];
    const float2 f0 = kf::unpack2<BF16>(v.x), f1 = kf::unpack2<BF16>(v.y);
    const float2 f2 = kf::unpack2<BF16>(v.z), f3 = kf::unpack2<BF16>(v.w);
    reinterpret_cast<float4*>(dst_o)[2 * i] = make_float4(f0.x, f0.y, f1.x, f1.y);
    reinterpret_cast<float4*>(dst_o)[2 * i + 1] = make_float4(f2.x, f2.y, f3.x, f3.y);
  }
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) h.lse[(int64_t)rank * rows + r] = lse[r];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    red_release_sys_add(h.counter, (uint32_t)(r1 - r0));
  }
}

// grid rows: merges the local split partials of one row (as merge_kernel) and
// sends the fp32 result to slot [rank] of every rank's mailbox.
__global__ void __launch_bounds__(kMergeThreads) merge_put_kernel(const MergeArgs a,
                                                                  const __grid_constant__ PeerSet peers,
                                                                  int world, int rank) {
  kf::griddep_wait();  // partials of the split kernel
  kf::griddep_launch_dependents();
  const PeerLayout L = peer_layout(world, a.rows, a.D);
  const uint32_t e = current_epoch(peers.mailbox[rank]);
  const int64_t row = blockIdx.x;
  const int64_t slot = (int64_t)rank * a.rows + row;
  merge_row_to(a, row, [&](int c4, float4 v, float l) {
    for (int p = 0; p < world; ++p) {
      const PeerHalf h = peer_half(peers.mailbox[p], L, e);
      *reinterpret_cast<float4*>(h.o + slot * a.D + c4 * 4) = v;
      if (c4 == 0) h.lse[slot] = l;
    }
  });
  // One signal per grid: every CTA orders its stores before its ticket
  // (gpu-scope fence); in the CTA that takes the last ticket, lane p of warp 0
  // releases all rows to receiver p: a system-scope fence, then a relaxed add
  // to p's arrival counter (fence + relaxed write is a release pattern).  The
  // receivers' fences run in parallel instead of one release per receiver in
  // turn, which grew the exchange with the rank count.
  __syncthreads();
  if (threadIdx.x < 32) {
    int last = 0;
    if (threadIdx.x == 0) {
      uint32_t* ticket = reinterpret_cast<uint32_t*>(peers.mailbox[rank]) + 2;
      __threadfence();
      last = atomicAdd(ticket, 1u) == gridDim.x - 1;
      if (last) *ticket = 0;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last && (int)threadIdx.x < world) {
      __threadfence_system();
      red_relaxed_sys_add(peer_half(peers.mailbox[threadIdx.x], L, e).counter, (uint32_t)a.rows);
    }
  }
}

// grid rows: waits (bounded) until all W x rows rows of this epoch arrived,
// merges one row, and the last CTA advances the epoch.
template <bool BF16>
__global__ void __launch_bounds__(kMergeThreads) peer_merge_kernel(MergeArgs m, uint8_t* mailbox,
                                                                    int world, int32_t* status) {
  __shared__ int s_ok;
  // the next kernel (a following decode call's split kernel) may set up while
  // this merge waits for the peers; it waits for this grid before any access
  kf::griddep_launch_dependents();
  const PeerLayout L = peer_layout(world, m.rows, m.D);
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(mailbox);
  const uint32_t e = current_epoch(mailbox);
  const PeerHalf h = peer_half(mailbox, L, e);
  if (threadIdx.x == 0) {
    const uint32_t target = (uint32_t)world * (uint32_t)m.rows * ((e + 1) >> 1);
    int ok = 1;
    const uint64_t t0 = kf::global_timer_ns();
    uint32_t spins = 0;
    while (ld_acquire_sys(h.counter) != target) {
      __nanosleep(32);
      if ((++spins & 255u) == 0 && kf::global_timer_ns() - t0 > kf::kWaitBudgetNs) {
        ok = 0;
        if (status) atomicExch(status, KF_DEV_TIMEOUT);
        break;
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  MergeArgs a = m;
  a.part_o = h.o;
  a.part_lse = h.lse;
  a.S = world;
  const int64_t row = blockIdx.x;
  if (s_ok) {
    merge_row<BF16>(a, row);
  } else {
    // a sender never arrived: NaN outputs instead of a partial merge
    merge_row_to(a, row, [&](int c4, float4, float) {
      const int64_t bh = row / a.Sq, s_ = row % a.Sq, b_ = bh / a.Hq, h_ = bh % a.Hq;
      uint16_t* dst = a.o + b_ * a.os0 + h_ * a.os1 + s_ * a.os2 + c4 * 4;
      *reinterpret_cast<uint2*>(dst) = make_uint2(0x7fff7fffu, 0x7fff7fffu);
      if (c4 == 0 && a.lse) a.lse[row] = __int_as_float(0x7fc00000);
    });
  }
  // every CTA has read the epoch before the last one takes its ticket
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ctrl + 1, 1u) == gridDim.x - 1) {
      ctrl[1] = 0;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(ctrl) = e;
    }
  }
}

typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddrRangeFn get_addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  });
  return fn;
}

int check_peer_shape(const char* what, int64_t rows, int64_t D, int dtype, int world) {
  if (world < 1 || world > kMaxPeers)
    return kf::set_error(KF_ERR_INVALID, "%s: need 1 <= world <= %d", what, kMaxPeers);
  if (rows <= 0 || rows > 0x7fffffffLL || D < 8 || D > 128 || D % 8)
    return kf::set_error(KF_ERR_INVALID, "%s: need rows > 0 and D a multiple of 8 in [8, 128]", what);
  if (dtype != KF_F16 && dtype != KF_BF16)
    return kf::set_error(KF_ERR_INVALID, "%s: dtype must be fp16 or bf16", what);
  return KF_OK;
}

bool misaligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }

int peer_set(const char* what, void* const* mailboxes, int world, int rank, PeerSet& peers) {
  if (!mailboxes) return kf::set_error(KF_ERR_INVALID, "%s: null mailboxes", what);
  if (rank < 0 || rank >= world) return kf::set_error(KF_ERR_INVALID, "%s: need 0 <= rank < world", what);
  peers = PeerSet{};
  for (int r = 0; r < world; ++r) {
    peers.mailbox[r] = static_cast<uint8_t*>(mailboxes[r]);
    if (!peers.mailbox[r] || misaligned(peers.mailbox[r], 256))
      return kf::set_error(KF_ERR_INVALID, "%s: mailboxes must be 256-byte aligned", what);
  }
  return KF_OK;
}

size_t merge_smem(int S, int D) {
  const int groups = kMergeThreads / (D / 4);
  return (size_t)(((S + 3) & ~3) + groups * D) * sizeof(float);
}

template <bool BF16>
int launch_peer_merge(const MergeArgs& m, uint8_t* mailbox, int world, int32_t* status, cudaStream_t st,
                      const char* what) {
  return launch_dependent(peer_merge_kernel<BF16>, dim3((unsigned)m.rows), dim3(kMergeThreads),
                          merge_smem(world, m.D), st, what, m, mailbox, world, status);
}

}  // namespace

extern "C" size_t kf_peer_mailbox_bytes(int world, int64_t rows, int64_t D) {
  if (world <= 0 || world > kMaxPeers || rows <= 0 || D <= 0) return 0;
  return (size_t)(256 + 2 * peer_layout(world, rows, (int)D).half);
}

extern "C" int kf_ipc_get_handle(const void* ptr, void* handle, uint64_t* offset) {
  using kf::set_error;
  if (!ptr || !handle || !offset) return set_error(KF_ERR_INVALID, "kf_ipc_get_handle: null argument");
  kf::DeviceGuard guard(ptr);
  if (guard.status()) return guard.status();

  AddrRangeFn range = get_addr_range_fn();
  if (!range) return set_error(KF_ERR_CUDA, "kf_ipc_get_handle: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(KF_ERR_INVALID, "kf_ipc_get_handle: pointer is not device memory");
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(KF_ERR_CUDA, "kf_ipc_get_handle: %s (the allocation must come from cudaMalloc)",
                     cudaGetErrorString(err));
  }
  memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<uint64_t>(ptr) - (uint64_t)base;
  return KF_OK;
}

extern "C" int kf_ipc_open_handle(const void* handle, uint64_t offset, void** ptr) {
  using kf::set_error;
  if (!handle || !ptr) return set_error(KF_ERR_INVALID, "kf_ipc_open_handle: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(KF_ERR_CUDA, "kf_ipc_open_handle: %s", cudaGetErrorString(err));
  }
  *ptr = static_cast<uint8_t*>(base) + offset;
  return KF_OK;
}

extern "C" int kf_ipc_close_handle(void* ptr, uint64_t offset) {
  if (!ptr) return kf::set_error(KF_ERR_INVALID, "kf_ipc_close_handle: null pointer");
  const cudaError_t err = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return kf::set_error(KF_ERR_CUDA, "kf_ipc_close_handle: %s", cudaGetErrorString(err));
  }
  return KF_OK;
}

extern "C" int kf_decode_peer_put(const void* o, const float* lse, int64_t rows, int64_t D, int dtype,
                                  void* const* mailboxes, int world, int rank, void* stream) {
  const char* what = "kf_decode_peer_put";
  if (!o || !lse) return kf::set_error(KF_ERR_INVALID, "%s: null argument", what);
  int rc = check_peer_shape(what, rows, D, dtype, world);
  if (rc) return rc;
  PeerSet peers;
  if ((rc = peer_set(what, mailboxes, world, rank, peers))) return rc;
  if (misaligned(o, 16) || misaligned(lse, 4)) return kf::set_error(KF_ERR_INVALID, "%s: misaligned buffers", what);
  kf::DeviceGuard guard(o);
  if (guard.status()) return guard.status();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rpp = put_rows_per_piece(rows, (int)D);
  const dim3 grid((unsigned)((rows + rpp - 1) / rpp), world);
  if (dtype == KF_BF16)
    peer_put_kernel<true><<<grid, kPeerThreads, 0, st>>>(static_cast<const uint16_t*>(o), lse, rows, (int)D, rpp,
                                                         peers, world, rank);
  else
    peer_put_kernel<false><<<grid, kPeerThreads, 0, st>>>(static_cast<const uint16_t*>(o), lse, rows, (int)D, rpp,
                                                          peers, world, rank);
  return kf::check_launch(what);
}

extern "C" int kf_decode_peer_merge(void* mailbox, int64_t rows, int64_t D, int dtype, int world, void* out,
                                    float* out_lse, int32_t* status, void* stream) {
  const char* what = "kf_decode_peer_merge";
  if (!mailbox || !out) return kf::set_error(KF_ERR_INVALID, "%s: null argument", what);
  int rc = check_peer_shape(what, rows, D, dtype, world);
  if (rc) return rc;
  if (misaligned(mailbox, 256) || misaligned(out, 8) || misaligned(out_lse, 4))
    return kf::set_error(KF_ERR_INVALID, "%s: misaligned buffers", what);
  kf::DeviceGuard guard(out);
  if (guard.status()) return guard.status();
  MergeArgs m = {};
  m.rows = rows;
  m.D = (int)D;
  m.o = static_cast<uint16_t*>(out);
  m.lse = out_lse;
  m.Hq = 1;
  m.Sq = 1;
  m.os0 = D;
  m.S = world;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* mb = static_cast<uint8_t*>(mailbox);
  return dtype == KF_BF16 ? launch_peer_merge<true>(m, mb, world, status, st, what)
                          : launch_peer_merge<false>(m, mb, world, status, st, what);
}

extern "C" int kf_decode_peer_exchange(const void* o, const float* lse, int64_t rows, int64_t D,
                                       int dtype, void* const* mailboxes, int world, int rank,
                                       void* out, float* out_lse, int32_t* status, void* stream) {
  if (!mailboxes || rank < 0 || rank >= world || world > kMaxPeers)
    return kf::set_error(KF_ERR_INVALID, "kf_decode_peer_exchange: need mailboxes and 0 <= rank < world <= %d",
                         kMaxPeers);
  int rc = kf_decode_peer_put(o, lse, rows, D, dtype, mailboxes, world, rank, stream);
  if (rc) return rc;
  return kf_decode_peer_merge(mailboxes[rank], rows, D, dtype, world, out, out_lse, status, stream);
}

namespace {

// Split kernel + merge_put (the send half of kf_decode_kv_split_peer); fills `local`.
int kv_split_send(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v, const kf_tensor4* o, float* lse,
                  int dtype, float scale, int num_splits, void* workspace, size_t workspace_bytes,
                  void* const* mailboxes, int world, int rank, cudaStream_t st, const char* what, PeerSet& peers,
                  MergeArgs& local) {
  if (num_splits < 1) return kf::set_error(KF_ERR_INVALID, "%s: num_splits must be >= 1", what);
  DecodeArgs a;
  int rc = decode_setup(q, k, v, nullptr, nullptr, 0, o, lse, dtype, scale, num_splits, workspace,
                        workspace_bytes, true, what, a);
  if (rc != KF_OK) return rc;
  if ((rc = check_peer_shape(what, a.prow_total, a.D, dtype, world))) return rc;
  if ((rc = peer_set(what, mailboxes, world, rank, peers))) return rc;
  if (a.num_splits > 2 * kMergeThreads)
    return kf::set_error(KF_ERR_UNSUPPORTED, "%s: at most %d splits", what, 2 * kMergeThreads);
  rc = dtype == KF_BF16 ? dispatch_split<true>(a, k, v, st) : dispatch_split<false>(a, k, v, st);
  if (rc != KF_OK) return rc;
  local = merge_args_of(a);
  const size_t smem = merge_smem(local.S, local.D);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(merge_put_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return kf::set_error(KF_ERR_CUDA, "%s: cannot reserve %zu bytes of shared memory", what, smem);
  return launch_dependent(merge_put_kernel, dim3((unsigned)local.rows), dim3(kMergeThreads), smem, st, what, local,
                          peers, world, rank);
}

}  // namespace

extern "C" int kf_decode_kv_split_peer_send(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                                            int dtype, float scale, int num_splits, void* workspace,
                                            size_t workspace_bytes, void* const* mailboxes, int world, int rank,
                                            void* stream) {
  if (!q) return kf::set_error(KF_ERR_INVALID, "kf_decode_kv_split_peer_send: null tensor descriptor");
  kf::DeviceGuard guard(q->ptr);
  if (guard.status()) return guard.status();
  PeerSet peers;
  MergeArgs local;
  // no output here: q stands in for O's descriptor (shape checks only)
  return kv_split_send(q, k, v, q, nullptr, dtype, scale, num_splits, workspace, workspace_bytes, mailboxes, world,
                       rank, static_cast<cudaStream_t>(stream), "kf_decode_kv_split_peer_send", peers, local);
}

extern "C" int kf_decode_kv_split_peer(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                                       const kf_tensor4* o, float* lse, int dtype, float scale, int num_splits,
                                       void* workspace, size_t workspace_bytes, void* const* mailboxes,
                                       int world, int rank, int32_t* status, void* stream) {
  const char* what = "kf_decode_kv_split_peer";
  if (!q) return kf::set_error(KF_ERR_INVALID, "%s: null tensor descriptor", what);
  kf::DeviceGuard guard(q->ptr);
  if (guard.status()) return guard.status();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  PeerSet peers;
  MergeArgs m;
  int rc = kv_split_send(q, k, v, o, lse, dtype, scale, num_splits, workspace, workspace_bytes, mailboxes, world,
                         rank, st, what, peers, m);
  if (rc != KF_OK) return rc;
  m.S = world;  // the final merge writes O/LSE with the caller's strides
  return dtype == KF_BF16 ? launch_peer_merge<true>(m, peers.mailbox[rank], world, status, st, what)
                          : launch_peer_merge<false>(m, peers.mailbox[rank], world, status, st, what);
}
