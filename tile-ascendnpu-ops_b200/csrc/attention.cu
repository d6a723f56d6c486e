// Flash-style attention forward on the 5th-generation tensor cores.
//
//   o   = softmax(scale * q k^T + mask) v        (per batch b, head h)
//   lse = log2(sum_j exp(scale * q.k_j))         (log2 domain, reference contract)
//
// Layout BSHD: q (B, Sq, H, D), k / v (B, Skv, Hkv, D), o like q, lse
// (B, H, Sq) fp32.  GQA: head h reads kv head h / (H / Hkv).  Causal masking
// is right-aligned: query i sees keys j <= i + Skv - Sq.
//
// Reference: kernels/attention/multi_head_attention/multi_head_attention_kernel/
// perf_opt/_gqa_prefill_fwd_kernel.py:199 (a two-phase kernel that writes S, P
// and the O partials to global workspaces) and its golden at :151-194.  Here S
// and P never leave the SM.
//
// One CTA computes two 128-row query tiles (t = 0, 1) of one (b, h) against
// the same stream of 128-key blocks, warp-specialised:
//   warps 0-3 / 4-7  softmax warpgroup of tile 0 / tile 1: thread r owns
//                    query row r of its tile (= TMEM lane r)
//   warp 8           TMA producer: Q0, Q1 once, then K_j / V_j (2-stage rings)
//   warp 9           MMA issuer (one thread) + TMEM owner
//   warps 10, 11     idle (they complete the third warpgroup, so that the
//                    register split below is the same on every SM
//                    sub-partition)
// setmaxnreg moves registers from the TMA / MMA warpgroup (72 each) to the
// softmax warpgroups (216 each), which hold a whole row of S.
// TMEM (512 columns): tile t uses [256t, 256t+128) for S_t, then P_t (bf16
// pairs, written over the first 64 columns once S_t is in registers), and
// [256t+128, 256t+128+D) for the O_t accumulator.
// Per block j the MMA thread issues, in order,
//   PV0_{j-1}: O0 += P0 V    (A = P from TMEM, B = V MN-major from smem)
//   S0_j     : S0 = Q0 K_j^T (A, B K-major from smem)
//   ... and the same for tile 1,
// so the tensor core works on one tile while the other tile's warpgroup runs
// its softmax.  tcgen05 ops of one thread complete in issue order, so the
// commit that signals "S_t,j done" also means "PV_t,j-1 done": the softmax
// warps may then rescale O_t in TMEM and overwrite S_t with P_t.
// Softmax: one TMEM pass puts the block's 128 scores of a row in registers;
// the running max moves (and O is rescaled) only when it grows by more than 8
// in log2 units, so P <= 256 and rescales are rare; exp2 is ex2.approx on
// exp2(scale*log2e*s - m), the FMA and the row sum as packed f32x2
// instructions; P is stored 32 scores at a time.
// Every mbarrier wait (sm100::mbar_wait) checks a 2 s limit between its
// try_wait polls: a phase that completes late ends the wait with an error
// (tileops_device_error_flag), and the kernel drains its copies / MMAs, frees
// TMEM and returns.  (A phase that never completes can park try_wait beyond
// the limit; none exists in this pipeline.)
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace tileops {
namespace {

using namespace sm100;

constexpr int kBM = 128;  // query rows per tile (two tiles per CTA)
constexpr int kTiles = 2;
constexpr int kBN = 128;  // keys per block
constexpr int kStages = 2;  // K and V ring depth
constexpr int kSoftmaxThreads = 128 * kTiles;
constexpr int kThreads = kSoftmaxThreads + 128;  // + one warpgroup: TMA, MMA, two idle warps
// Register split (setmaxnreg): launched at kLaunchRegs per thread, the
// TMA / MMA warpgroup gives registers back and the softmax warpgroups take
// them, so a softmax thread holds a whole row of S.  Per SM sub-partition
// (one warp of each warpgroup): 2 x 216 + 72 = 3 x 168.
constexpr int kLaunchRegs = 168;
constexpr int kSoftmaxRegs = 216;
constexpr int kProducerRegs = 72;
static_assert(kTiles * 4 * kSoftmaxRegs + 4 * kProducerRegs == (kThreads / 32) * kLaunchRegs,
              "register split must equal the launch allocation");
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kGroupBH = 16;  // (b, h) pairs per launch-order group

template <int D>
struct Smem {
  static constexpr int kTile = kBM * D * 2;  // bytes of a 128 x D 16-bit tile
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTiles * kTile;
  static constexpr int kV = kK + kStages * kTile;
  static constexpr int kBar = kV + kStages * kTile;
  static constexpr int kBytes = kBar + 256;
  static constexpr int kAlloc = kBytes + 1024;  // room to align the base to 1024
};

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[kTiles], p_full[kTiles], o_done[kTiles];
  uint64_t mma_drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct Params {
  int batch, heads, heads_kv, seq_q, seq_kv;
  float scale_log2;  // sm_scale * log2(e)
  int causal;
  void* o;
  float* lse;
  int* err;
};

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  if (bf16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Number of key blocks query tile starting at q0 needs.
__device__ __forceinline__ int tile_blocks(int q0, const Params& p) {
  if (q0 >= p.seq_q) return 0;
  int kv_end = p.seq_kv;
  if (p.causal) kv_end = min(kv_end, min(q0 + kBM, p.seq_q) - 1 + (p.seq_kv - p.seq_q) + 1);
  return kv_end > 0 ? (kv_end + kBN - 1) / kBN : 0;
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using L = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + L::kBar);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_ct = (p.seq_q + kTiles * kBM - 1) / (kTiles * kBM);
  // CTAs start in linear grid order.  That order walks groups of kGroupBH
  // (b, h) pairs; inside a group the longest (causal) query tiles of all its
  // pairs come first, so the grid ends on short CTAs while the K / V of the
  // few pairs in flight stay in L2.
  const int nbh = static_cast<int>(gridDim.y);
  const int lin = static_cast<int>(blockIdx.y) * num_ct + static_cast<int>(blockIdx.x);
  const int grp = lin / (kGroupBH * num_ct);
  const int gsz = min(kGroupBH, nbh - grp * kGroupBH);
  const int within = lin - grp * kGroupBH * num_ct;
  const int ct = num_ct - 1 - within / gsz;
  const int bh = grp * kGroupBH + within % gsz;
  const int b = bh / p.heads;
  const int h = bh - b * p.heads;
  const int hk = h / (p.heads / p.heads_kv);
  const int q_cta = ct * kTiles * kBM;
  int nb[kTiles];
#pragma unroll
  for (int t = 0; t < kTiles; ++t) nb[t] = tile_blocks(q_cta + t * kBM, p);
  const int nblk = max(nb[0], nb[1]);

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 128);
      mbar_init(&bars->o_done[t], 1);
    }
    mbar_init(&bars->mma_drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  constexpr uint32_t kTileBytes = L::kTile;
  constexpr int kChunks = D / 64;  // 64-wide (128-byte) column chunks of a tile

  if (warp >= 8) reg_dealloc<kProducerRegs>();
  if (warp == 8) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0 && nblk > 0) {
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
      mbar_arrive_expect_tx(&bars->q_full, kTiles * kTileBytes);
      for (int t = 0; t < kTiles; ++t)
        for (int c = 0; c < kChunks; ++c)
          tma_load_4d(smem + L::kQ + t * kTileBytes + c * (kBM * 128), &tm_q, &bars->q_full,
                      c * 64, h, q_cta + t * kBM, b);
      int armed_k = -1, armed_v = -1;
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kStages;
        const uint32_t use = j / kStages;
        if (use > 0 && !mbar_wait(&bars->k_empty[s], (use - 1) & 1, p.err, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->k_full[s], kTileBytes);
        for (int c = 0; c < kChunks; ++c)
          tma_load_4d(smem + L::kK + s * kTileBytes + c * (kBN * 128), &tm_k, &bars->k_full[s],
                      c * 64, hk, j * kBN, b);
        armed_k = j;
        if (use > 0 && !mbar_wait(&bars->v_empty[s], (use - 1) & 1, p.err, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->v_full[s], kTileBytes);
        for (int c = 0; c < kChunks; ++c)
          tma_load_4d(smem + L::kV + s * kTileBytes + c * (kBN * 128), &tm_v, &bars->v_full[s],
                      c * 64, hk, j * kBN, b);
        armed_v = j;
      }
      // Drain: never leave the CTA with a bulk copy still writing its smem.
      mbar_wait(&bars->q_full, 0, p.err, abort_flag, true);
      if (armed_k >= 0)
        mbar_wait(&bars->k_full[armed_k % kStages], (armed_k / kStages) & 1, p.err, abort_flag,
                  true);
      if (armed_v >= 0)
        mbar_wait(&bars->v_full[armed_v % kStages], (armed_v / kStages) & 1, p.err, abort_flag,
                  true);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t idesc_qk = idesc_f16(kBM, kBN, BF16 ? 1 : 0, 0);
      constexpr uint32_t idesc_pv = idesc_f16(kBM, D, BF16 ? 1 : 0, 1);
      bool ok = mbar_wait(&bars->q_full, 0, p.err, abort_flag);
      // Descriptors of the tile bases, built once; every k-step's descriptor
      // is one of these advanced by a compile-time byte offset.
      const uint64_t q_desc = smem_desc(smem_u32(smem + L::kQ), 16, 1024);
      const uint64_t k_desc = smem_desc(smem_u32(smem + L::kK), 16, 1024);
      const uint64_t v_desc = smem_desc(smem_u32(smem + L::kV), kBN * 128, 1024);
      auto issue_s = [&](int t, int j) {  // S_t = Q_t K_j^T
        const uint64_t qd = desc_advance(q_desc, t * kTileBytes);
        const uint64_t kd = desc_advance(k_desc, (j % kStages) * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off_b = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
          mma_f16_ss(tmem + t * 256, desc_advance(qd, off_b), desc_advance(kd, off_b), idesc_qk,
                     kk > 0);
        }
        mma_commit(&bars->s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {  // O_t += P_t V_j
        const uint64_t vd = desc_advance(v_desc, (j % kStages) * kTileBytes);
        const uint32_t t_p = tmem + t * 256;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          mma_f16_ts(t_p + 128, t_p + kk * 8, desc_advance(vd, kk * 16 * 128), idesc_pv,
                     (j > 0 || kk > 0));
      };
      // Prologue: S for block 0 of both tiles.
      if (ok) ok = mbar_wait(&bars->k_full[0], 0, p.err, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < kTiles; ++t)
          if (nb[t] > 0) issue_s(t, 0);
        mma_commit(&bars->k_empty[0]);
      }
      for (int j = 0; ok && j < nblk; ++j) {
        if (!mbar_wait(&bars->v_full[j % kStages], (j / kStages) & 1, p.err, abort_flag)) break;
        const bool more = j + 1 < nblk;
        if (more && !mbar_wait(&bars->k_full[(j + 1) % kStages], ((j + 1) / kStages) & 1, p.err,
                               abort_flag))
          break;
        for (int t = 0; t < kTiles; ++t) {
          if (j >= nb[t]) continue;
          if (!mbar_wait(&bars->p_full[t], j & 1, p.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_pv(t, j);
          if (j + 1 < nb[t]) issue_s(t, j + 1);
          else mma_commit(&bars->o_done[t]);
        }
        if (!ok) break;
        mma_commit(&bars->v_empty[j % kStages]);
        if (more) mma_commit(&bars->k_empty[(j + 1) % kStages]);
      }
      // Drain: every MMA this thread issued completes before TMEM is freed.
      mma_commit(&bars->mma_drain);
      mbar_wait(&bars->mma_drain, 0, p.err, abort_flag, true);
    }
  } else if (warp < 8) {
    // ------------------------------------- softmax warpgroups (warps 0..7)
    reg_alloc<kSoftmaxRegs>();
    const int t = warp >> 2;                 // tile of this warpgroup
    const int row = threadIdx.x & 127;       // row within the tile == TMEM lane
    const int q0 = q_cta + t * kBM;
    const int q_idx = q0 + row;
    const int n_t = nb[t];
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_base + t * 256;  // S / P columns of this row
    const uint32_t t_o = t_s + 128;                   // O columns of this row
    const int off = p.seq_kv - p.seq_q;
    const int row_limit = p.causal ? q_idx + off : p.seq_kv - 1;  // last visible key
    const float sl2 = p.scale_log2;
    float m = -INFINITY;  // running max, log2-scaled units
    float l = 0.0f;       // running sum of exp2(x - m)
    bool ok = true;
    for (int j = 0; j < n_t; ++j) {
      if (!mbar_wait(&bars->s_full[t], j & 1, p.err, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int k0 = j * kBN;
      const bool need_mask = (k0 + kBN > p.seq_kv) || (p.causal && k0 + kBN - 1 > q0 + off);
      // Keys this row may see in the block: [k0, k0 + nvis).
      const int nvis = need_mask ? max(0, min(kBN, min(p.seq_kv - 1, row_limit) + 1 - k0)) : kBN;
      // The block's scores of this row, all four 32-column loads in flight at once.
      uint32_t sc[kBN / 32][32];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) tmem_ld32(t_s + c * 32, sc[c]);
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) tmem_wait_ld_regs(sc[c]);
      // Row max of the raw scores (scale > 0 commutes with max), 8 chains.
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
      if (!need_mask) {  // two scores per three-input max
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
          for (int i = 0; i < 16; ++i)
            mx[i & 7] = fmax3(mx[i & 7], __uint_as_float(sc[c][2 * i]),
                              __uint_as_float(sc[c][2 * i + 1]));
      } else {
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i < nvis) mx[i & 7] = fmaxf(mx[i & 7], __uint_as_float(sc[c][i]));
      }
      const float mraw = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      const float mloc = mraw * sl2;
      float m_use = m;
      if (mloc > m + kRescaleThreshold || m == -INFINITY) m_use = fmaxf(mloc, m);
      const float m_sub = (m_use == -INFINITY) ? 0.0f : m_use;
      const float m_prev = m;
      m = m_use;
      // O_t is idle here (PV_t,j-1 completed before S_t,j; PV_t,j waits for
      // this block's P): rescale the rows whose max moved.  The whole warp
      // takes the branch (tcgen05.ld / st are .sync.aligned); alpha = 1 leaves
      // the other rows as they are.
      if (j > 0 && __any_sync(0xffffffffu, m_use != m_prev)) {
        const float alpha = m_use != m_prev ? ex2(m_prev - m_use) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(t_o + c * 32, r);
          tmem_wait_ld_regs(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(t_o + c * 32, r);
        }
        l *= alpha;
      }
      // P = exp2(scale*log2e*s - m) two scores at a time (packed f32x2 FMA
      // and add), packed to 16-bit pairs over S columns [0, 64).
      float2 ps[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
      {
        const float2 scale2 = make_float2(sl2, sl2), negm2 = make_float2(-m_sub, -m_sub);
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int kk = c * 32 + 2 * i;
            const float2 x = ffma2(
                make_float2(__uint_as_float(sc[c][2 * i]), __uint_as_float(sc[c][2 * i + 1])),
                scale2, negm2);
            float e0 = ex2(x.x), e1 = ex2(x.y);
            if (need_mask) {
              e0 = kk < nvis ? e0 : 0.0f;
              e1 = kk + 1 < nvis ? e1 : 0.0f;
            }
            ps[i & 1] = fadd2(ps[i & 1], make_float2(e0, e1));
            pk[i] = pack2(e0, e1, BF16);
          }
          tmem_st16(t_s + c * 16, pk);
        }
      }
      const float rowsum = (ps[0].x + ps[1].x) + (ps[0].y + ps[1].y);
      l += rowsum;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[t]);
    }
    // Epilogue: O / l -> o, lse = m + log2(l).
    if (ok && n_t > 0 && mbar_wait(&bars->o_done[t], 0, p.err, abort_flag)) {
      tc_fence_after();
      const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      T* orow = static_cast<T*>(p.o) +
                ((static_cast<int64_t>(b) * p.seq_q + q_idx) * p.heads + h) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_o + c * 32, r);
        tmem_wait_ld_regs(r);
        if (q_idx < p.seq_q) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 v;
            v.x = pack2(__uint_as_float(r[u * 8 + 0]) * inv_l, __uint_as_float(r[u * 8 + 1]) * inv_l, BF16);
            v.y = pack2(__uint_as_float(r[u * 8 + 2]) * inv_l, __uint_as_float(r[u * 8 + 3]) * inv_l, BF16);
            v.z = pack2(__uint_as_float(r[u * 8 + 4]) * inv_l, __uint_as_float(r[u * 8 + 5]) * inv_l, BF16);
            v.w = pack2(__uint_as_float(r[u * 8 + 6]) * inv_l, __uint_as_float(r[u * 8 + 7]) * inv_l, BF16);
            *reinterpret_cast<uint4*>(orow + c * 32 + u * 8) = v;
          }
        }
      }
      if (q_idx < p.seq_q)
        p.lse[(static_cast<int64_t>(b) * p.heads + h) * p.seq_q + q_idx] =
            l > 0.0f ? m + log2f(l) : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host
template <int D, bool BF16>
int launch_attn(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H,
                int Hkv, int Sq, int Skv, int causal, float sm_scale, cudaStream_t s) {
  CUtensorMap tq, tk, tv;
  if (!make_bshd_map(&tq, q, D, H, Sq, B, 128, BF16) ||
      !make_bshd_map(&tk, k, D, Hkv, Skv, B, 128, BF16) ||
      !make_bshd_map(&tv, v, D, Hkv, Skv, B, 128, BF16))
    return TILEOPS_ELAUNCH;
  Params p;
  p.batch = B;
  p.heads = H;
  p.heads_kv = Hkv;
  p.seq_q = Sq;
  p.seq_kv = Skv;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.causal = causal;
  p.o = o;
  p.lse = lse;
  p.err = device_error_ptr();
  auto kern = attn_fwd_kernel<D, BF16>;
  const int smem = Smem<D>::kAlloc;
  // The setmaxnreg split assumes exactly kLaunchRegs registers per thread at
  // launch; with fewer the increases could never be granted.
  static const bool regs_ok = [kern] {
    cudaFuncAttributes a;
    return cudaFuncGetAttributes(&a, kern) == cudaSuccess && a.numRegs == kLaunchRegs;
  }();
  if (!regs_ok) return TILEOPS_ELAUNCH;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return TILEOPS_ELAUNCH;
  dim3 grid((Sq + kTiles * kBM - 1) / (kTiles * kBM), B * H);
  kern<<<grid, kThreads, smem, s>>>(tq, tk, tv, p);
  return launch_status();
}

}  // namespace
}  // namespace tileops

using namespace tileops;

extern "C" int tileops_mha_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                               int64_t batch, int64_t heads, int64_t heads_kv, int64_t seq_q,
                               int64_t seq_kv, int64_t dim, int is_causal, double sm_scale,
                               int dtype, void* stream) {
  if (batch < 0 || heads <= 0 || heads_kv <= 0 || seq_q < 0 || seq_kv < 0)
    return TILEOPS_EBADSHAPE;
  if (heads % heads_kv != 0) return TILEOPS_EBADSHAPE;
  if (dim != 64 && dim != 128) return TILEOPS_EBADSHAPE;
  if (is_causal && seq_q > seq_kv) return TILEOPS_EBADSHAPE;
  if (batch * heads > 65535 || seq_q > (1 << 30) || seq_kv > (1 << 30)) return TILEOPS_EBADSHAPE;
  // The kernel numbers its CTAs with a 32-bit linear index.
  if ((seq_q + kTiles * kBM - 1) / (kTiles * kBM) * batch * heads > 0x7fffffffLL)
    return TILEOPS_EBADSHAPE;
  if (dtype != TILEOPS_DT_BF16 && dtype != TILEOPS_DT_F16) return TILEOPS_EBADDTYPE;
  if (batch == 0 || seq_q == 0) return TILEOPS_OK;
  if (seq_kv == 0) return TILEOPS_EBADSHAPE;  // no key to attend to
  if (!q || !k || !v || !o || !lse) return TILEOPS_EINVAL;
  // TMA: 16-byte aligned base addresses (every stride is a multiple of 16 B).
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return TILEOPS_EALIGN;
  cudaStream_t s = as_stream(stream);
  const bool bf16 = dtype == TILEOPS_DT_BF16;
  const int B = static_cast<int>(batch), H = static_cast<int>(heads),
            Hkv = static_cast<int>(heads_kv), Sq = static_cast<int>(seq_q),
            Skv = static_cast<int>(seq_kv);
  const float sc = static_cast<float>(sm_scale);
  if (dim == 128)
    return bf16 ? launch_attn<128, true>(q, k, v, o, lse, B, H, Hkv, Sq, Skv, is_causal, sc, s)
                : launch_attn<128, false>(q, k, v, o, lse, B, H, Hkv, Sq, Skv, is_causal, sc, s);
  return bf16 ? launch_attn<64, true>(q, k, v, o, lse, B, H, Hkv, Sq, Skv, is_causal, sc, s)
              : launch_attn<64, false>(q, k, v, o, lse, B, H, Hkv, Sq, Skv, is_causal, sc, s);
}
