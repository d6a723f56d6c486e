// Gated DeltaNet (gated delta rule) chunked prefill.
//
// Recurrence per (batch b, head h), token t, state S (dk x dv, fp32):
//   S <- exp(g_t) S ;  S <- S + k_t (x) beta_t (v_t - k_t^T S) ;  o_t = scale q_t^T S
// (reference golden: examples/gdn_prefill/probe/gdn_prefill_probe.py:60-77;
// chunk algebra: the same file :19-26 and examples/gdn_prefill/DESIGN.md).
//
// Chunked form (chunk of C = 64 tokens, S the state at the chunk start,
// gc = inclusive cumulative sum of g inside the chunk, G[l,s] = exp(gc_l - gc_s)):
//   A[l,s]  = beta_l G[l,s] (k_l . k_s)        l > s    (strictly lower)
//   T       = (I + A)^-1                         (unit lower triangular)
//   Wk      = T (beta e^gc (.) K)                C x dk   } S-independent:
//   U       = T (beta (.) V)                     C x dv   } computed for every
//   QKm     = scale G (.) (Q K^T), l >= s        C x C    } chunk in parallel
//   err     = U - Wk S                           (the per-token beta(v - k^T S))
//   o       = scale e^gc (.) (Q S) + QKm err
//   S_next  = e^gc_last S + K^T (e^(gc_last - gc) (.) err)
//
// Kernel 1 (gdn_prepare): one CTA per (b, h, chunk), K / Q / V by TMA.
// KK^T and QK^T on tensor cores (mma.sync bf16, fp32 accumulate, lower
// triangle only); T by 16 x 16 block forward substitution in fp32 (diagonal
// blocks by substitution, off-diagonal blocks by T_ij = -T_ii sum_m A_im T_mj,
// one warp per block); Wk = (T diag(beta e^gc)) K and U = (T diag(beta)) V as
// tensor-core products.  Results go to a caller-provided workspace,
// 64 x (dk + dv + 64) bf16 plus 132 fp32 per chunk.
// Kernel 2 (gdn_scan): one CTA per (b, h, 64-wide slice of dv) -- the columns
// of S evolve independently -- walking the chunks in order.  S lives in fp32
// registers as MMA accumulators; one thread streams every chunk's operands
// (q, k and the workspace tiles) one chunk ahead by TMA into swizzled shared
// memory.
//
// Layout: q, k (B, T, H, dk) bf16; v, o (B, T, H, dv) bf16; g, beta (B, T, H)
// fp32; initial / final state (B, H, dk, dv) fp32.
//
// Sequences.  Both kernels see the tokens as rows: B sequences of T rows for
// a uniform batch; for variable-length input one packed axis where sequence
// n is rows [cu_seqlens[n], cu_seqlens[n+1]) (the fla varlen convention,
// batch 1).  A chunk is 64 rows of one sequence; the rows of its last chunk
// past the sequence end are padding: their g and beta read as 0 and their k,
// q, v rows are zero (TMA zero fill past T for a uniform batch; for variable
// length they hold the next sequence's tokens and are zeroed in shared memory
// after the load), so they leave the state unchanged; their outputs are not
// stored.  Chunk slots: sequence n with nc_n chunks owns the slots
// [base_n, base_n + nc_n), base_n = n * nchunks for a uniform batch and
// base_n = floor(cu[n] / 64) + n for variable length (disjoint ranges for a
// non-decreasing cu, all below nslots = floor(total / 64) + N); chunk c of
// head h is workspace unit H base_n + h nc_n + c (for a uniform batch the
// (b, h, chunk) order, consecutive units = consecutive chunks of one head).
#include <mutex>
#include <vector>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace tileops {
namespace {

constexpr int kC = 64;  // chunk length

// ---------------------------------------------------- warp-level MMA helpers
__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr(p)));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// B fragments of two adjacent n-tiles (n0.., n0+8..) where B[k][n] is stored
// row-major [k][n]: b[0..1] for tile n0, b[2..3] for tile n0 + 8.
__device__ __forceinline__ void frag_b_kn(uint32_t (&b)[4], const __nv_bfloat16* base, int ld,
                                          int k0, int n0) {
  const int lane = threadIdx.x & 31;
  const int mat = lane >> 3;  // 0: (k0,n0) 1: (k0+8,n0) 2: (k0,n0+8) 3: (k0+8,n0+8)
  ldsm_x4_t(b, base + (k0 + (lane & 7) + ((mat & 1) << 3)) * ld + n0 + ((mat >> 1) << 3));
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Workspace of one chunk (element offsets into a bf16 array, then fp32 tail).
template <int DK, int DV>
struct Ws {
  static constexpr int64_t kWk = 0;                 // C x DK bf16, holds -Wk
  static constexpr int64_t kU = kWk + kC * DK;      // C x DV bf16
  static constexpr int64_t kQK = kU + kC * DV;      // C x C bf16
  static constexpr int64_t kHalfs = kQK + kC * kC;  // bf16 elements before the fp32 tail
  // fp32 tail (fp32 element offsets from the chunk start):
  static constexpr int64_t kQsc = kHalfs / 2;   // C: scale * exp(gc_l)
  static constexpr int64_t kDec = kQsc + kC;    // C: exp(gc_last - gc_l)
  static constexpr int64_t kEgl = kDec + kC;    // 1: exp(gc_last) (+3 padding)
  static constexpr int kTailFloats = 2 * kC + 4;
  static constexpr int64_t kBytes = kHalfs * 2 + kTailFloats * 4;  // multiple of 16
};

// Where the sequences of one call lie on the flat token axis.
struct SeqLayout {
  const int* cu;         // nullptr: uniform batch; else N + 1 row offsets
  const int* chunk_seq;  // variable length: the sequence whose slot range holds slot j
  int rows;              // uniform: tokens per sequence; variable: total rows
  int nchunks;           // uniform: chunks per sequence
  int nslots;            // chunk slots per head
};

// TMA coordinates (row, batch) of row t of sequence n: the (D, H, T, B) map
// of a uniform batch, the (D, H, total, 1) map of packed sequences.
// kVar: packed sequences (sl.cu set); the kernels are instantiated for both
// forms so a uniform batch carries none of the variable-length logic.
template <bool kVar>
__device__ __forceinline__ int2 map_row(int n, int bos, int t) {
  if constexpr (kVar) return make_int2(t, 0);
  else return make_int2(t - bos, n);
}

// Rows [bos, eos) of sequence n and its first chunk slot.  Variable-length
// offsets are clamped into [0, rows] (and eos >= bos), so a malformed
// cu_seqlens can give wrong numbers but never an out-of-range access; the
// index kernel reports it.
template <bool kVar>
__device__ __forceinline__ void seq_span(const SeqLayout& sl, int n, int& bos, int& eos,
                                         int& base) {
  if constexpr (!kVar) {
    bos = n * sl.rows;
    eos = bos + sl.rows;
    base = n * sl.nchunks;
  } else {
    bos = min(max(sl.cu[n], 0), sl.rows);
    eos = min(max(sl.cu[n + 1], bos), sl.rows);
    base = (bos >> 6) + n;
  }
}

// Variable length: chunk_seq[j] = the largest n with base_n <= j (the
// sequence whose slot range [base_n, base_n+1) holds slot j).  Threads n < N
// also check the offsets (cu[0] = 0, cu[N] = rows, non-decreasing) and report
// kErrBadSeqlens otherwise.
__global__ void gdn_chunk_index(SeqLayout sl, int nseq, int* __restrict__ chunk_seq, int* err) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  const int* cu = sl.cu;
  if (j < nseq) {
    const bool bad = cu[j] > cu[j + 1] || (j == 0 && cu[0] != 0) ||
                     (j == nseq - 1 && cu[nseq] != sl.rows);
    if (bad) report_device_error(err, kErrBadSeqlens);
  }
  if (j >= sl.nslots) return;
  int lo = 0, hi = nseq - 1;  // invariant: base_lo <= j (base_0 = 0)
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    const int bos = min(max(cu[mid], 0), sl.rows);
    if ((bos >> 6) + mid <= j) lo = mid;
    else hi = mid - 1;
  }
  chunk_seq[j] = lo;
}

// =========================================================== kernel 1
// 128 threads (4 warps), one CTA per (b, h, chunk); four CTAs per SM.
// K, Q, V arrive by TMA as 128-byte-swizzled [64][64] bf16 boxes (tokens
// past T read as zeros).  Shared memory:
//   Ks [64][DK]                swizzled bf16 (TMA)
//   Qs [64][DK]                swizzled bf16 (TMA); once QK^T is formed the
//                              region holds Tf (T in fp32, [64][68]) and then
//                              Tk, Tv (swizzled bf16 [64][64] each)
//   As fp32 [64][65]           A, strictly lower; once T is formed the region
//                              takes V (swizzled [64][DV] bf16, TMA)
//   gc, beta, ke = beta e^gc   [64] each
//   mbarrier + abort flag
// Tile addressing: 16-byte unit u of row r in a 64-column box at
// ((u ^ (r & 7)) << 4), boxes 8 KB apart.
__device__ __forceinline__ uint32_t swz(int r, int col) {  // col % 8 == 0
  return ((col >> 6) << 13) + (r << 7) + ((((col & 63) >> 3) ^ (r & 7)) << 4);
}
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// The four fragment loaders of the padded tiles, for swizzled tiles at
// shared address `base` (same lane -> (row, column) assignment).
__device__ __forceinline__ void sfrag_a(uint32_t (&a)[4], uint32_t base, int m0, int k0) {
  const int lane = threadIdx.x & 31;
  ldsm4(a, base + swz(m0 + (lane & 15), k0 + ((lane >> 4) << 3)));
}
__device__ __forceinline__ void sfrag_a_t(uint32_t (&a)[4], uint32_t base, int m0, int k0) {
  const int lane = threadIdx.x & 31, mat = lane >> 3;
  ldsm4t(a, base + swz(k0 + (lane & 7) + ((mat >> 1) << 3), m0 + ((mat & 1) << 3)));
}
__device__ __forceinline__ void sfrag_b_kn(uint32_t (&b)[4], uint32_t base, int k0, int n0) {
  const int lane = threadIdx.x & 31, mat = lane >> 3;
  ldsm4t(b, base + swz(k0 + (lane & 7) + ((mat & 1) << 3), n0 + ((mat >> 1) << 3)));
}
__device__ __forceinline__ void sfrag_b_nk(uint32_t (&b)[4], uint32_t base, int k0, int n0) {
  const int lane = threadIdx.x & 31, mat = lane >> 3;
  ldsm4(b, base + swz(n0 + (lane & 7) + ((mat >> 1) << 3), k0 + ((mat & 1) << 3)));
}

// Zeroes rows first..63 of `boxes` swizzled [64][64] bf16 boxes (8 KB apart);
// a row is 128 contiguous bytes whatever the swizzle.  Called by every thread
// of the CTA (strided over blockDim.x).
__device__ __forceinline__ void zero_rows(uint8_t* tile, int boxes, int first) {
  const int per_box = (kC - first) * 8;  // 16-byte units
  for (int i = threadIdx.x; i < boxes * per_box; i += blockDim.x) {
    const int bx = i / per_box, rem = i - bx * per_box;
    *reinterpret_cast<uint4*>(tile + bx * 8192 + (first + (rem >> 3)) * 128 + (rem & 7) * 16) =
        make_uint4(0u, 0u, 0u, 0u);
  }
}

constexpr int kLdTf = 68;  // fp32 row stride of Tf (16-byte aligned rows)
constexpr int kLdA = 65;   // fp32 row stride of As

template <int DK, int DV>
struct PrepSmem {
  static constexpr int cmax(int a, int b) { return a > b ? a : b; }
  static constexpr int kKs = 0;
  static constexpr int kQs = kKs + kC * DK * 2;
  static constexpr int kQsBytes = cmax(cmax(kC * DK * 2, kC * kLdTf * 4), 2 * kC * kC * 2);
  // As (fp32 [64][65]) until T is formed, then V (swizzled [64][DV] bf16).
  static constexpr int kAs = (kQs + kQsBytes + 1023) & ~1023;
  static constexpr int kVs = kAs;
  static constexpr int kGc = kAs + cmax(kC * kLdA * 4, kC * DV * 2);
  static constexpr int kBeta = kGc + kC * 4;
  static constexpr int kKe = kBeta + kC * 4;
  static constexpr int kEgp = kKe + kC * 4;     // e^gc
  static constexpr int kEgm = kEgp + kC * 4;    // e^-gc, and the factor flag after it
  static constexpr int kRk = kEgm + kC * 4 + 16;  // 1 / |k_l| (fused q/k L2 norm)
  static constexpr int kRq = kRk + kC * 4;        // 1 / |q_l|
  // two mbarriers, the abort flag, then the chunk's (map row, map batch,
  // head, first row to zero) read back late instead of held in registers
  static constexpr int kBar = kRq + kC * 4;
  static constexpr int kBytes = kBar + 48;
  static constexpr int kAlloc = kBytes + 1024;  // room to align the base to 1 KB
};

template <int DK, int DV, bool kVar, bool kNorm>
__global__ void __launch_bounds__(128, 4)
    gdn_prepare(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_wk,
                const __grid_constant__ CUtensorMap tm_u, const float* __restrict__ g,
                const float* __restrict__ beta, __nv_bfloat16* __restrict__ ws, SeqLayout sl,
                int H, float scale, int* err) {
  using L = PrepSmem<DK, DV>;
  using W = Ws<DK, DV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = saddr(sm);
  float* As = reinterpret_cast<float*>(sm + L::kAs);
  float* Tf = reinterpret_cast<float*>(sm + L::kQs);
  float* gc = reinterpret_cast<float*>(sm + L::kGc);
  float* bt = reinterpret_cast<float*>(sm + L::kBeta);
  float* ke = reinterpret_cast<float*>(sm + L::kKe);
  float* egp = reinterpret_cast<float*>(sm + L::kEgp);
  float* egm = reinterpret_cast<float*>(sm + L::kEgm);
  int* fact_flag = reinterpret_cast<int*>(sm + L::kEgm + kC * 4);
  float* rk = reinterpret_cast<float*>(sm + L::kRk);
  float* rq = reinterpret_cast<float*>(sm + L::kRq);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::kBar);       // K, Q
  uint64_t* bar_v = reinterpret_cast<uint64_t*>(sm + L::kBar + 8);  // V
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::kBar + 16);
  int* chunk_info = reinterpret_cast<int*>(sm + L::kBar + 32);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t2 = (lane & 3) * 2;
  // CTA = workspace unit u = H base_n + h nc_n + c.
  const int u = blockIdx.x;
  const int n = kVar ? sl.chunk_seq[u / H] : u / (H * sl.nchunks);
  int bos, eos, base;
  seq_span<kVar>(sl, n, bos, eos, base);
  const int nc = kVar ? (eos - bos + kC - 1) / kC : sl.nchunks;
  const int r = u - H * base;
  if constexpr (kVar) {
    if (r < 0 || r >= H * nc) return;  // a unit past the sequence's chunks
  }
  const int h = r / nc;
  const int t0 = bos + (r - h * nc) * kC;  // first row of the chunk
  const int nvalid = min(kC, eos - t0);   // rows of this sequence in it
  const int zpad = kVar ? nvalid : kC;  // first row to zero after a load
  const int2 mrow = map_row<kVar>(n, bos, t0);
  __nv_bfloat16* wsc = ws + static_cast<int64_t>(blockIdx.x) * (W::kBytes / 2);
  float* wsf = reinterpret_cast<float*>(wsc);

  if (tid == 0) {
    sm100::mbar_init(bar, 1);
    sm100::mbar_init(bar_v, 1);
    *abort_flag = 0;
    chunk_info[0] = mrow.x;
    chunk_info[1] = mrow.y;
    chunk_info[2] = h;
    chunk_info[3] = zpad;
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    sm100::mbar_arrive_expect_tx(bar, 2 * DK * kC * 2);
#pragma unroll
    for (int c = 0; c < DK / 64; ++c) {
      sm100::tma_load_4d(sm + L::kKs + c * 8192, &tm_k, bar, c * 64, h, mrow.x, mrow.y);
      sm100::tma_load_4d(sm + L::kQs + c * 8192, &tm_q, bar, c * 64, h, mrow.x, mrow.y);
    }
  }
  if (warp == 0) {
    // inclusive cumsum of g over the 64 tokens: two per lane + warp scan
    float g0 = 0.0f, g1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
    if (2 * lane < nvalid) {
      const int64_t o = static_cast<int64_t>(t0 + 2 * lane) * H + h;
      g0 = g[o];
      b0 = beta[o];
    }
    if (2 * lane + 1 < nvalid) {
      const int64_t o = static_cast<int64_t>(t0 + 2 * lane + 1) * H + h;
      g1 = g[o];
      b1 = beta[o];
    }
    const float pair = g0 + g1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float up = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += up;
    }
    const float excl = incl - pair;
    const float c0 = excl + g0, c1 = incl;
    gc[2 * lane] = c0;
    gc[2 * lane + 1] = c1;
    bt[2 * lane] = b0;
    bt[2 * lane + 1] = b1;
    // G[l, s] = e^(gc_l - gc_s) may be formed as e^gc_l * e^-gc_s when every
    // |gc| of the chunk is below 80 (both factors then stay finite in fp32).
    float amax = fmaxf(fabsf(c0), fabsf(c1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    egp[2 * lane] = __expf(c0);
    egp[2 * lane + 1] = __expf(c1);
    egm[2 * lane] = __expf(-c0);
    egm[2 * lane + 1] = __expf(-c1);
    if (lane == 0) *fact_flag = amax < 80.0f ? 1 : 0;
  }
  // Every thread waits for the tiles (bounded); the CTA proceeds only if all
  // saw them land, otherwise it lets any copy in flight finish and leaves.
  const bool landed = sm100::mbar_wait(bar, 0, err, abort_flag);
  if (!__syncthreads_and(landed)) {
    if (tid == 0) sm100::mbar_wait(bar, 0, nullptr, abort_flag, true);
    __syncthreads();
    return;
  }
  const uint32_t sK = sb + L::kKs, sQ = sb + L::kQs, sV = sb + L::kVs;
  if (zpad < kC) {  // padding rows of K and Q -> 0
    zero_rows(sm + L::kKs, DK / 64, zpad);
    zero_rows(sm + L::kQs, DK / 64, zpad);
    __syncthreads();
  }
  if constexpr (kNorm) {
    // Fused q / k L2 norm: 1 / sqrt(sum x^2 + 1e-6) per row (thread t: row
    // t % 64 of K for t < 64, of Q otherwise).  Nothing is rewritten; the
    // factors scale the products and the per-row workspace tail below.
    const int row = tid & 63;
    const uint8_t* tile = sm + (tid < 64 ? L::kKs : L::kQs) + row * 128;
    float ss = 0.0f;
#pragma unroll
    for (int bx = 0; bx < DK / 64; ++bx)
#pragma unroll
      for (int u8 = 0; u8 < 8; ++u8) {
        const uint4 pk = *reinterpret_cast<const uint4*>(tile + bx * 8192 + u8 * 16);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h2[e]);
          ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
        }
      }
    (tid < 64 ? rk : rq)[row] = 1.0f / sqrtf(ss + 1e-6f);
    __syncthreads();
  }

  // ---- KK^T -> A (strictly lower, fp32) and QK^T -> QKm (lower, bf16, to the
  // workspace); warp w owns rows 16w..16w+15 and only needs columns <= them.
  {
    const int m0 = warp * 16;
    const int ntiles = 2 * (warp + 1);
    float ak[8][4], aq[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) ak[n][e] = aq[n][e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
      uint32_t fk[4], fq[4];
      sfrag_a(fk, sK, m0, kk * 16);
      sfrag_a(fq, sQ, m0, kk * 16);
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        if (n < ntiles) {
          uint32_t bb[4];
          sfrag_b_nk(bb, sK, kk * 16, n * 8);
          mma_bf16(ak[n], fk, bb[0], bb[1]);
          mma_bf16(ak[n + 1], fk, bb[2], bb[3]);
          mma_bf16(aq[n], fq, bb[0], bb[1]);
          mma_bf16(aq[n + 1], fq, bb[2], bb[3]);
        }
      }
    }
    const bool fact = *fact_flag != 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int l = m0 + g8 + half * 8;
      const float gl = gc[l], bl = bt[l], el = egp[l];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int s = n * 8 + t2;
        float d0, d1;
        if (fact) {
          d0 = s <= l ? el * egm[s] : 0.0f;
          d1 = s + 1 <= l ? el * egm[s + 1] : 0.0f;
        } else {
          d0 = s <= l ? __expf(gl - gc[s]) : 0.0f;
          d1 = s + 1 <= l ? __expf(gl - gc[s + 1]) : 0.0f;
        }
        if constexpr (kNorm) {  // k_l . k_s / (|k_l| |k_s|), q_l . k_s / (|q_l| |k_s|)
          const float rkl = rk[l], rql = rq[l], rk0 = rk[s], rk1 = rk[s + 1];
          ak[n][half * 2] *= rkl * rk0;
          ak[n][half * 2 + 1] *= rkl * rk1;
          aq[n][half * 2] *= rql * rk0;
          aq[n][half * 2 + 1] *= rql * rk1;
        }
        As[l * kLdA + s] = s < l ? bl * d0 * ak[n][half * 2] : 0.0f;
        As[l * kLdA + s + 1] = s + 1 < l ? bl * d1 * ak[n][half * 2 + 1] : 0.0f;
        *reinterpret_cast<uint32_t*>(wsc + W::kQK + l * kC + s) =
            pack_bf16(scale * d0 * aq[n][half * 2], scale * d1 * aq[n][half * 2 + 1]);
      }
    }
  }
  __syncthreads();  // As complete; the Qs region is free for Tf

  // ---- diagonal 16 x 16 blocks of T = (I + A)^-1 by forward substitution
  // (threads 0..63: one column each); threads 64..127 write the fp32 tail
  // of the workspace and ke = beta e^gc.
  if (tid < 64) {
    const int blk = tid >> 4, col = tid & 15, base = blk * 16;
    float t[16];
#pragma unroll
    for (int l = 0; l < 16; ++l) {
      float acc = 0.0f;
#pragma unroll
      for (int m = 0; m < l; ++m) acc = fmaf(As[(base + l) * kLdA + base + m], t[m], acc);
      t[l] = (l == col) ? 1.0f : (l > col ? -acc : 0.0f);
    }
#pragma unroll
    for (int l = 0; l < 16; ++l) Tf[(base + l) * kLdTf + base + col] = t[l];
  } else {
    const int i = tid - 64;
    const float gl = gc[kC - 1];
    const float e = __expf(gc[i]);
    // With the fused norm, 1/|k_i| joins the factors that multiply row i of K
    // (Wk = T diag(ke) K here, K^T (dec err) in the scan) and 1/|q_i| the one
    // that multiplies row i of Q S.
    const float nk = kNorm ? rk[i] : 1.0f, nq = kNorm ? rq[i] : 1.0f;
    ke[i] = bt[i] * e * nk;
    wsf[W::kQsc + i] = scale * e * nq;
    wsf[W::kDec + i] = __expf(gl - gc[i]) * nk;
    if (i < 4) wsf[W::kEgl + i] = i == 0 ? __expf(gl) : 0.0f;
  }
  __syncthreads();

  // ---- off-diagonal blocks by distance d = i - j: warp p < 4 - d forms
  //   X = sum_{m=j}^{i-1} A_im T_mj,   T_ij = -T_ii X      ((i, j) = (p + d, p))
  // in fp32 on the CUDA cores; lane -> row lane / 2, columns 8 (lane % 2)...
#pragma unroll
  for (int d = 1; d < 4; ++d) {
    if (warp < 4 - d) {
      const int i = warp + d, j = warp;
      const int r = lane >> 1, c0 = j * 16 + (lane & 1) * 8;
      float x[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = 0.0f;
#pragma unroll
      for (int mm = 0; mm < d; ++mm) {
        const int m = j + mm;
#pragma unroll
        for (int kx = 0; kx < 16; ++kx) {
          const float a = As[(i * 16 + r) * kLdA + m * 16 + kx];
          const float4 u = *reinterpret_cast<const float4*>(Tf + (m * 16 + kx) * kLdTf + c0);
          const float4 w = *reinterpret_cast<const float4*>(Tf + (m * 16 + kx) * kLdTf + c0 + 4);
          x[0] = fmaf(a, u.x, x[0]);
          x[1] = fmaf(a, u.y, x[1]);
          x[2] = fmaf(a, u.z, x[2]);
          x[3] = fmaf(a, u.w, x[3]);
          x[4] = fmaf(a, w.x, x[4]);
          x[5] = fmaf(a, w.y, x[5]);
          x[6] = fmaf(a, w.z, x[6]);
          x[7] = fmaf(a, w.w, x[7]);
        }
      }
      float* xo = Tf + (i * 16 + r) * kLdTf + c0;  // block (i, j) holds X for now
      *reinterpret_cast<float4*>(xo) = make_float4(x[0], x[1], x[2], x[3]);
      *reinterpret_cast<float4*>(xo + 4) = make_float4(x[4], x[5], x[6], x[7]);
      __syncwarp();
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = 0.0f;
#pragma unroll
      for (int kx = 0; kx < 16; ++kx) {
        const float a = Tf[(i * 16 + r) * kLdTf + i * 16 + kx];
        const float4 u = *reinterpret_cast<const float4*>(Tf + (i * 16 + kx) * kLdTf + c0);
        const float4 w = *reinterpret_cast<const float4*>(Tf + (i * 16 + kx) * kLdTf + c0 + 4);
        y[0] = fmaf(a, u.x, y[0]);
        y[1] = fmaf(a, u.y, y[1]);
        y[2] = fmaf(a, u.z, y[2]);
        y[3] = fmaf(a, u.w, y[3]);
        y[4] = fmaf(a, w.x, y[4]);
        y[5] = fmaf(a, w.y, y[5]);
        y[6] = fmaf(a, w.z, y[6]);
        y[7] = fmaf(a, w.w, y[7]);
      }
      __syncwarp();
      *reinterpret_cast<float4*>(xo) = make_float4(-y[0], -y[1], -y[2], -y[3]);
      *reinterpret_cast<float4*>(xo + 4) = make_float4(-y[4], -y[5], -y[6], -y[7]);
    }
    __syncthreads();
  }
  // As is dead: V lands in its place while Tk, Tv and Wk are formed.
  if (tid == 0) {
    sm100::fence_proxy_async_smem();
    sm100::mbar_arrive_expect_tx(bar_v, DV * kC * 2);
#pragma unroll
    for (int c = 0; c < DV / 64; ++c)
      sm100::tma_load_4d(sm + L::kVs + c * 8192, &tm_v, bar_v, c * 64, chunk_info[2],
                         chunk_info[0], chunk_info[1]);
  }

  // ---- Tk = T diag(beta e^gc), Tv = T diag(beta) in bf16, swizzled [64][64]
  // each, over the Tf region (read all of Tf first).
  {
    const int l = tid >> 1, s0 = (tid & 1) * 32;
    float tv[32];
#pragma unroll
    for (int q4 = 0; q4 < 8; ++q4) {
      const float4 u = *reinterpret_cast<const float4*>(Tf + l * kLdTf + s0 + q4 * 4);
      tv[q4 * 4 + 0] = u.x;
      tv[q4 * 4 + 1] = u.y;
      tv[q4 * 4 + 2] = u.z;
      tv[q4 * 4 + 3] = u.w;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 pk, pv;
      uint32_t* pkw = reinterpret_cast<uint32_t*>(&pk);
      uint32_t* pvw = reinterpret_cast<uint32_t*>(&pv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int s = s0 + c * 8 + 2 * e;
        const float v0 = s <= l ? tv[c * 8 + 2 * e] : 0.0f;
        const float v1 = s + 1 <= l ? tv[c * 8 + 2 * e + 1] : 0.0f;
        pkw[e] = pack_bf16(v0 * ke[s], v1 * ke[s + 1]);
        pvw[e] = pack_bf16(v0 * bt[s], v1 * bt[s + 1]);
      }
      *reinterpret_cast<uint4*>(sm + L::kQs + swz(l, s0 + c * 8)) = pk;
      *reinterpret_cast<uint4*>(sm + L::kQs + 8192 + swz(l, s0 + c * 8)) = pv;
    }
  }
  __syncthreads();

  // ---- Wk = Tk K (C x DK), then (once V has landed) U = Tv V (C x DV): warp
  // w owns output columns [w D/4, (w+1) D/4) of all four 16-row blocks; T is
  // lower triangular, so row block m takes k-blocks 0..m (every warp the same
  // ten (m, k) pairs: the work is balanced across the warps).  Each
  // result is staged in shared memory (swizzled [64][64] boxes, the freed K
  // tile for -Wk, the freed Tk / Tv tile for U) and written by TMA stores, so
  // the workspace sees whole 128-byte lines.
  {
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      if (which == 1) {
        const bool v_landed = sm100::mbar_wait(bar_v, 0, err, abort_flag);
        if (!__syncthreads_and(v_landed)) {
          if (tid == 0) {
            sm100::mbar_wait(bar_v, 0, nullptr, abort_flag, true);
            sm100::bulk_wait_read_all();
          }
          __syncthreads();
          return;
        }
        if (chunk_info[3] < kC) {  // padding rows of V -> 0
          zero_rows(sm + L::kVs, DV / 64, chunk_info[3]);
          __syncthreads();
        }
      }
      constexpr int kMaxD = DK > DV ? DK : DV;
      constexpr int kMaxNT = kMaxD / 32;  // 8-column tiles per warp
      const int D = which == 0 ? DK : DV;
      const int NT = D / 32;
      const int cw = warp * NT * 8;  // first output column of this warp
      const uint32_t tA = sb + L::kQs + which * 8192;
      const uint32_t X = which == 0 ? sK : sV;
      float acc[4][kMaxNT][4];
#pragma unroll
      for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int n = 0; n < kMaxNT; ++n)
          acc[m][n][0] = acc[m][n][1] = acc[m][n][2] = acc[m][n][3] = 0.0f;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
#pragma unroll
        for (int kk = 0; kk <= m; ++kk) {
          uint32_t a[4];
          sfrag_a(a, tA, m * 16, kk * 16);
#pragma unroll
          for (int n = 0; n < kMaxNT; n += 2) {
            if (n >= NT) break;
            uint32_t bb[4];
            sfrag_b_kn(bb, X, kk * 16, cw + n * 8);
            mma_bf16(acc[m][n], a, bb[0], bb[1]);
            mma_bf16(acc[m][n + 1], a, bb[2], bb[3]);
          }
        }
      }
      __syncthreads();  // every read of the tile the result is staged into is done
      // The workspace keeps -Wk (the scans add it) and U.
      uint8_t* stage = sm + (which == 0 ? L::kKs : L::kQs);
      const float sg = which == 0 ? -1.0f : 1.0f;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
#pragma unroll
        for (int n = 0; n < kMaxNT; ++n) {
          if (n >= NT) break;
          const int l = m * 16 + g8, col = cw + n * 8;  // swz() adds the 64-column box
          *reinterpret_cast<uint32_t*>(stage + swz(l, col) + t2 * 2) =
              pack_bf16(sg * acc[m][n][0], sg * acc[m][n][1]);
          *reinterpret_cast<uint32_t*>(stage + swz(l + 8, col) + t2 * 2) =
              pack_bf16(sg * acc[m][n][2], sg * acc[m][n][3]);
        }
      }
      sm100::fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) {
        for (int nb = 0; nb * 64 < D; ++nb)
          sm100::tma_store_3d(which == 0 ? &tm_wk : &tm_u, stage + nb * 8192, nb * 64, 0,
                              static_cast<int>(blockIdx.x));
        sm100::bulk_commit();
      }
    }
    if (tid == 0) sm100::bulk_wait_read_all();  // shared memory stays valid until read
  }
}

// =========================================================== kernel 2
// 256 threads (8 warps), one CTA per (b, h, 64-column slice of dv), walking
// the chunks in order.  Thread 0 streams every chunk's operands one chunk
// ahead by TMA into two stages of 128-byte-swizzled tiles:
//   Qs, Ks, Wks [64][DK]; Us [64][64] (the slice of U); QKs [64][64];
//   the workspace's fp32 tail (a plain bulk copy).
// Besides the stages: Ss [DK][72] (S in bf16, the B operand of Wk S and
// Q S), Es / Ed [64][72] (err and decayed err, B operands), padded.
constexpr int kSlice = 64;

template <int DK>
struct ScanSmem {
  static constexpr int kLdS = kSlice + 8;
  static constexpr int kQs = 0;
  static constexpr int kKs = kQs + kC * DK * 2;
  static constexpr int kWks = kKs + kC * DK * 2;
  static constexpr int kUs = kWks + kC * DK * 2;
  static constexpr int kQKs = kUs + kC * kSlice * 2;
  static constexpr int kEg = kQKs + kC * kC * 2;  // the workspace fp32 tail
  static constexpr int kTailBytes = (2 * kC + 4) * 4;
  static constexpr int kStage = (kEg + kTailBytes + 1023) & ~1023;
  static constexpr int kLoadBytes = 3 * kC * DK * 2 + kC * kSlice * 2 + kC * kC * 2 + kTailBytes;
  static constexpr int kSs = 2 * kStage;
  static constexpr int kEs = kSs + DK * kLdS * 2;
  static constexpr int kEd = kEs + kC * kLdS * 2;
  static constexpr int kBar = kEd + kC * kLdS * 2;  // full[2] + abort flag
  static constexpr int kBytes = kBar + 32;
  static constexpr int kAlloc = kBytes + 1024;
};

template <int DK, int DV, bool kVar>
__global__ void __launch_bounds__(256, 1)
    gdn_scan(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
             const __grid_constant__ CUtensorMap tm_wk, const __grid_constant__ CUtensorMap tm_u,
             const __grid_constant__ CUtensorMap tm_qk, const __nv_bfloat16* __restrict__ ws,
             const float* __restrict__ h0, __nv_bfloat16* __restrict__ o, float* __restrict__ hT,
             SeqLayout sl, int H, int* err) {
  using L = ScanSmem<DK>;
  using W = Ws<DK, DV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = saddr(sm);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kSlices = DV / kSlice;
  const int slice = blockIdx.x % kSlices;
  const int bh = blockIdx.x / kSlices;
  const int b = bh / H, h = bh - (bh / H) * H;  // b: the sequence
  const int v0 = slice * kSlice;
  const int g8 = lane >> 2, t2 = (lane & 3) * 2;
  int bos, eos, base;
  seq_span<kVar>(sl, b, bos, eos, base);
  const int nchunks = kVar ? (eos - bos + kC - 1) / kC : sl.nchunks;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::kBar);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::kBar + 16);

  auto issue = [&](int s, int chunk) {  // thread 0 only
    const int t0 = bos + chunk * kC;
    const int unit = H * base + h * nchunks + chunk;  // workspace chunk unit
    const int2 mrow = map_row<kVar>(b, bos, t0);
    uint8_t* st = sm + s * L::kStage;
    sm100::mbar_arrive_expect_tx(&full[s], L::kLoadBytes);
#pragma unroll
    for (int c = 0; c < DK / 64; ++c) {
      sm100::tma_load_4d(st + L::kQs + c * 8192, &tm_q, &full[s], c * 64, h, mrow.x, mrow.y);
      sm100::tma_load_4d(st + L::kKs + c * 8192, &tm_k, &full[s], c * 64, h, mrow.x, mrow.y);
      sm100::tma_load_3d(st + L::kWks + c * 8192, &tm_wk, &full[s], c * 64, 0, unit);
    }
    sm100::tma_load_3d(st + L::kUs, &tm_u, &full[s], v0, 0, unit);
    sm100::tma_load_3d(st + L::kQKs, &tm_qk, &full[s], 0, 0, unit);
    sm100::bulk_load(st + L::kEg,
                     reinterpret_cast<const float*>(ws + static_cast<int64_t>(unit) * (W::kBytes / 2)) +
                         W::kQsc,
                     L::kTailBytes, &full[s]);
  };

  __nv_bfloat16* Ss = reinterpret_cast<__nv_bfloat16*>(sm + L::kSs);
  __nv_bfloat16* Es = reinterpret_cast<__nv_bfloat16*>(sm + L::kEs);
  __nv_bfloat16* Ed = reinterpret_cast<__nv_bfloat16*>(sm + L::kEd);

  if (tid == 0) {
    sm100::mbar_init(&full[0], 1);
    sm100::mbar_init(&full[1], 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0 && nchunks > 0) issue(0, 0);

  // State: warp w owns rows 16w..16w+15 of S (DK = 128: rows 0..127) as
  // 8 n-tiles of 16 x 8 accumulators (the 64-column slice).
  constexpr int kRowTiles = DK / 16;  // == 8 for DK = 128, 4 for DK = 64
  const bool owns_rows = warp < kRowTiles;
  const int sr0 = warp * 16;
  float S[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float val = 0.0f;
      if (owns_rows && h0) {
        const int r = sr0 + g8 + ((e >> 1) << 3), c = n * 8 + t2 + (e & 1);
        val = h0[((static_cast<int64_t>(b) * H + h) * DK + r) * DV + v0 + c];
      }
      S[n][e] = val;
    }
  auto publish_state = [&]() {  // S (fp32 regs) -> Ss (bf16 B operand [DK][64])
    if (!owns_rows) return;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int r = sr0 + g8, c = n * 8 + t2;
      *reinterpret_cast<uint32_t*>(Ss + r * L::kLdS + c) = pack_bf16(S[n][0], S[n][1]);
      *reinterpret_cast<uint32_t*>(Ss + (r + 8) * L::kLdS + c) = pack_bf16(S[n][2], S[n][3]);
    }
  };
  publish_state();

  // Output tiles: warp w -> rows 16(w%4).., columns 32(w/4).. of the 64 x 64 o slice.
  const int om0 = (warp & 3) * 16, on0 = (warp >> 2) * 32;
  int failed_at = -1;

  for (int chunk = 0; chunk < nchunks; ++chunk) {
    const int s = chunk & 1;
    // Stage s^1 was released by the barrier that ended the previous chunk.
    if (tid == 0 && chunk + 1 < nchunks) issue(s ^ 1, chunk + 1);
    const bool landed = sm100::mbar_wait(&full[s], (chunk >> 1) & 1, err, abort_flag);
    if (!__syncthreads_and(landed)) {  // also: the published state is visible
      failed_at = chunk;
      break;
    }
    const int nvalid = min(kC, eos - (bos + chunk * kC));
    if (kVar && nvalid < kC) {  // padding rows of K -> 0 (they enter K^T err)
      zero_rows(sm + s * L::kStage + L::kKs, DK / 64, nvalid);
      sm100::fence_proxy_async_smem();  // before the stage's next TMA refill
      __syncthreads();
    }
    const uint32_t st = sb + s * L::kStage;
    const uint32_t sQ = st + L::kQs, sK = st + L::kKs, sW = st + L::kWks;
    const uint32_t sU = st + L::kUs, sQK = st + L::kQKs;
    const uint8_t* Ub = sm + s * L::kStage + L::kUs;
    const float* egs = reinterpret_cast<const float*>(sm + s * L::kStage + L::kEg);
    const float* qsc = egs;            // scale * exp(gc_l)
    const float* dcy = egs + kC;       // exp(gc_last - gc_l)
    const float egl = egs[2 * kC];     // exp(gc_last)
    // err = U - Wk S (the workspace holds -Wk) ; qs = Q S   (this warp's 16 x 32 tile)
    float ws_acc[4][4], qs_acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) ws_acc[n][e] = qs_acc[n][e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
      uint32_t aw[4], aq[4];
      sfrag_a(aw, sW, om0, kk * 16);
      sfrag_a(aq, sQ, om0, kk * 16);
#pragma unroll
      for (int n = 0; n < 4; n += 2) {
        uint32_t bb[4];
        frag_b_kn(bb, Ss, L::kLdS, kk * 16, on0 + n * 8);
        mma_bf16(ws_acc[n], aw, bb[0], bb[1]);
        mma_bf16(ws_acc[n + 1], aw, bb[2], bb[3]);
        mma_bf16(qs_acc[n], aq, bb[0], bb[1]);
        mma_bf16(qs_acc[n + 1], aq, bb[2], bb[3]);
      }
    }
    float o_acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int l = om0 + g8 + half * 8, c = on0 + n * 8 + t2;
        const __nv_bfloat162 u2 =
            *reinterpret_cast<const __nv_bfloat162*>(Ub + swz(l, c - t2) + t2 * 2);
        const float e0 = __bfloat162float(u2.x) + ws_acc[n][half * 2];  // U + (-Wk) S
        const float e1 = __bfloat162float(u2.y) + ws_acc[n][half * 2 + 1];
        const float dec = dcy[l];
        *reinterpret_cast<uint32_t*>(Es + l * L::kLdS + c) = pack_bf16(e0, e1);
        *reinterpret_cast<uint32_t*>(Ed + l * L::kLdS + c) = pack_bf16(dec * e0, dec * e1);
        o_acc[n][half * 2] = qsc[l] * qs_acc[n][half * 2];
        o_acc[n][half * 2 + 1] = qsc[l] * qs_acc[n][half * 2 + 1];
      }
    }
    __syncthreads();  // err published; every read of Ss for this chunk is done
    // o += QKm err  (QKm lower triangular: k-blocks 0 .. this warp's row block)
    for (int kk = 0; kk <= (warp & 3); ++kk) {
      uint32_t a[4];
      sfrag_a(a, sQK, om0, kk * 16);
#pragma unroll
      for (int n = 0; n < 4; n += 2) {
        uint32_t bb[4];
        frag_b_kn(bb, Es, L::kLdS, kk * 16, on0 + n * 8);
        mma_bf16(o_acc[n], a, bb[0], bb[1]);
        mma_bf16(o_acc[n + 1], a, bb[2], bb[3]);
      }
    }
    {
      const int t0 = bos + chunk * kC;
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int l = om0 + g8 + half * 8, c = on0 + n * 8 + t2;
          if (l < nvalid)
            *reinterpret_cast<uint32_t*>(o + (static_cast<int64_t>(t0 + l) * H + h) * DV + v0 +
                                         c) = pack_bf16(o_acc[n][half * 2],
                                                        o_acc[n][half * 2 + 1]);
        }
    }
    // S = e^gc_last S + K^T (decayed err)
    if (owns_rows) {
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[n][e] *= egl;
#pragma unroll
      for (int kk = 0; kk < kC / 16; ++kk) {
        uint32_t a[4];
        sfrag_a_t(a, sK, sr0, kk * 16);
#pragma unroll
        for (int n = 0; n < 8; n += 2) {
          uint32_t bb[4];
          frag_b_kn(bb, Ed, L::kLdS, kk * 16, n * 8);
          mma_bf16(S[n], a, bb[0], bb[1]);
          mma_bf16(S[n + 1], a, bb[2], bb[3]);
        }
      }
    }
    __syncthreads();  // Es / Ed and this stage are free; Ss may be rewritten
    publish_state();
  }
  if (failed_at >= 0) {
    // A wait gave up: let the copies already issued (this chunk's and the
    // next one's) land before leaving.
    if (tid == 0)
      for (int c = failed_at; c < failed_at + 2 && c < nchunks; ++c)
        sm100::mbar_wait(&full[c & 1], (c >> 1) & 1, nullptr, abort_flag, true);
    __syncthreads();
    return;
  }
  if (owns_rows && hT) {
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = sr0 + g8 + ((e >> 1) << 3), c = n * 8 + t2 + (e & 1);
        hT[((static_cast<int64_t>(b) * H + h) * DK + r) * DV + v0 + c] = S[n][e];
      }
  }
}

// =========================================================== kernel 2b
// gdn_scan_tc: the chunk scan on the 5th-generation tensor cores (dk = 128).
// One CTA per (b, h, 64-column slice of dv), 320 threads:
//   warps 0-7  math: warp w serves TMEM lanes 32 (w % 4).. (rows of every
//              accumulator) and columns 32 (w / 4).. of the 64-wide slice
//   warp 8     TMA producer (two stages, one chunk ahead)
//   warp 9     MMA issuer (one thread) and TMEM owner (512 columns)
// TMEM: D1 x3 [128 x 64] at columns 0 / 64 / 128, D2 x2 at 192 / 256, the
// state S [128 x 64] at 320.
// Per chunk c (S the state at the chunk start, Sb its bf16 copy in smem; the
// workspace holds -Wk):
//   MMA0  D1 = [I ; 0] U            (no dependence on S: issued early)
//   MMA1  D1 += [-Wk ; Q] Sb        (rows 0-63: err = U - Wk S, 64-127: Q S)
//   math  Es = err, Ed = e^(gc_last - gc) err (bf16)           (rows 0-63)
//   MMA3  S += K^T Ed               (S pre-scaled by e^gc_last), commit
//   MMA2  D2 = [U ; QKm] Es         (rows 64-127: QKm err)
//   math  S -> Sb (bf16), S *= e^(gc_last of chunk c+1)   -> next chunk
//   math  o = scale e^gc (Q S) + QKm err   (rows 64-127, off the chain)
// The chain from one chunk to the next is MMA1, the err pass (Ed only: Es
// follows on its own barrier for MMA2), MMA3 and the state pass (up to the
// bf16 copy Sb: the pre-scaled TMEM copy is written after s_ready, since only
// MMA3 of the next chunk, which waits for e_ready, reads it); D1 is triple-
// and D2 double-buffered so the output pass of chunk c overlaps chunk c+1.
// Shared memory per stage (128-byte swizzled tiles, 64 KB): A1 = [-Wk ; Q]
// as two chunks of [128][64]; K [64][128]; [U ; QKm] as one [128][64] tile
// (the B operand of MMA0 is its U half; as the A operand of MMA2 its U rows
// only feed rows of D2 that are never read).  Outside the stages: the
// identity tile [I ; 0], the fp32 tails, Sb [128][64] (MN-major B of MMA1),
// Es, Ed [64][64] (MN-major B of MMA2 / MMA3).
constexpr int kTcStages = 2;
struct ScanTcSmem {
  static constexpr int kA1 = 0;                           // 2 x 16 KB
  static constexpr int kK = kA1 + 2 * 16384;              // 2 x 8 KB
  static constexpr int kUQ = kK + 2 * 8192;               // U 8 KB, then QKm 8 KB
  static constexpr int kStage = kUQ + 16384;              // 64 KB
  static constexpr int kTailBytes = (2 * kC + 4) * 4;
  static constexpr int kLoadBytes = 2 * 8192 /*Wk*/ + 2 * 8192 /*Q*/ + 2 * 8192 /*K*/ +
                                    8192 /*U*/ + 8192 /*QKm*/ + kTailBytes;
  static constexpr int kId = kTcStages * kStage;          // 16 KB
  static constexpr int kSb = kId + 16384;                 // 16 KB
  static constexpr int kEs = kSb + 16384;                 // 8 KB
  static constexpr int kEd = kEs + 8192;                  // 8 KB
  static constexpr int kTail = kEd + 8192;                // kTcStages x 528 B
  static constexpr int kBar = kTail + kTcStages * kTailBytes;
  static constexpr int kBytes = kBar + 128;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 232448, "scan_tc shared memory exceeds 227 KB");
};

struct ScanTcBars {
  uint64_t full[kTcStages], empty[kTcStages];
  uint64_t s_ready, d1_full, e_ready, es_ready, d3_full, d2_full, drain;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr int kScanTcMath = 256;
constexpr int kScanTcThreads = kScanTcMath + 64;
constexpr uint32_t kScanTcCols = 512;

template <int DV, bool kVar>
__global__ void __launch_bounds__(kScanTcThreads, 1)
    gdn_scan_tc(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_wk,
                const __grid_constant__ CUtensorMap tm_u,
                const __grid_constant__ CUtensorMap tm_qk, const __nv_bfloat16* __restrict__ ws,
                const float* __restrict__ h0, __nv_bfloat16* __restrict__ o,
                float* __restrict__ hT, SeqLayout sl, int H, int* err) {
  using namespace sm100;
  using L = ScanTcSmem;
  using W = Ws<128, DV>;
  constexpr int DK = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  ScanTcBars* bars = reinterpret_cast<ScanTcBars*>(sm + L::kBar);
  volatile int* abort_flag = &bars->abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int kSlices = DV / kSlice;
  const int slice = blockIdx.x % kSlices;
  const int bh = blockIdx.x / kSlices;
  const int b = bh / H, h = bh - (bh / H) * H;  // b: the sequence
  const int v0 = slice * kSlice;
  int bos, eos, base;
  seq_span<kVar>(sl, b, bos, eos, base);
  const int nchunks = kVar ? (eos - bos + kC - 1) / kC : sl.nchunks;
  if (kVar && nchunks == 0) {  // an empty sequence: the final state is the initial one
    if (hT != nullptr)
      for (int i = tid; i < DK * kSlice; i += blockDim.x) {
        const int64_t at = ((static_cast<int64_t>(b) * H + h) * DK + i / kSlice) * DV + v0 +
                           i % kSlice;
        hT[at] = h0 ? h0[at] : 0.0f;
      }
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->s_ready, kScanTcMath);
    mbar_init(&bars->d1_full, 1);
    mbar_init(&bars->e_ready, kScanTcMath);
    mbar_init(&bars->es_ready, kScanTcMath / 2);
    mbar_init(&bars->d3_full, 1);
    mbar_init(&bars->d2_full, 1);
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&bars->tmem_base, kScanTcCols);
    tmem_relinquish();
  }
  if (tid < kScanTcMath) {
    // The identity tile [I ; 0]: 128 rows x 64 bf16, K-major, swizzled.
    for (int i = tid; i < 128 * 8; i += kScanTcMath) {
      const int r = i >> 3, u = i & 7;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < 64 && (r >> 3) == u) {
        uint32_t* vw = reinterpret_cast<uint32_t*>(&v);
        vw[(r & 7) >> 1] = (r & 1) ? 0x3F800000u : 0x00003F80u;  // bf16 1.0 at column r
      }
      *reinterpret_cast<uint4*>(sm + L::kId + swz(r, 8 * u)) = v;
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t t_s = tmem + 320;
  auto t_d1 = [&](int c) { return tmem + 64u * static_cast<uint32_t>(c % 3); };
  auto t_d2 = [&](int c) { return tmem + 192u + 64u * static_cast<uint32_t>(c & 1); };

  if (warp == 8) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_wk);
      prefetch_tensormap(&tm_u);
      prefetch_tensormap(&tm_qk);
      int armed = -1;
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % kTcStages;
        const int use = c / kTcStages;
        if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, err, abort_flag)) break;
        uint8_t* st = sm + s * L::kStage;
        const int t0 = bos + c * kC;
        const int unit = H * base + h * nchunks + c;
        const int2 mrow = map_row<kVar>(b, bos, t0);
        mbar_arrive_expect_tx(&bars->full[s], L::kLoadBytes);
#pragma unroll
        for (int k = 0; k < DK / 64; ++k) {
          tma_load_3d(st + L::kA1 + k * 16384, &tm_wk, &bars->full[s], k * 64, 0, unit);
          tma_load_4d(st + L::kA1 + k * 16384 + 8192, &tm_q, &bars->full[s], k * 64, h, mrow.x,
                      mrow.y);
          tma_load_4d(st + L::kK + k * 8192, &tm_k, &bars->full[s], k * 64, h, mrow.x, mrow.y);
        }
        tma_load_3d(st + L::kUQ, &tm_u, &bars->full[s], v0, 0, unit);
        tma_load_3d(st + L::kUQ + 8192, &tm_qk, &bars->full[s], 0, 0, unit);
        bulk_load(sm + L::kTail + s * L::kTailBytes,
                  reinterpret_cast<const float*>(ws + static_cast<int64_t>(unit) * (W::kBytes / 2)) +
                      W::kQsc,
                  L::kTailBytes, &bars->full[s]);
        armed = c;
      }
      // Never leave with a bulk copy still writing this CTA's shared memory.
      for (int c = armed - (kTcStages - 1); c <= armed; ++c)
        if (c >= 0)
          mbar_wait(&bars->full[c % kTcStages], (c / kTcStages) & 1, err, abort_flag, true);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_kmn = idesc_f16_major(128, 64, 1, 0, 1);  // A K-major, B MN-major
      constexpr uint32_t id_mnmn = idesc_f16_major(128, 64, 1, 1, 1);  // A MN-major (K^T)
      // Base descriptors built once; k-steps advance them by constant offsets.
      const uint64_t id_d = smem_desc(smem_u32(sm + L::kId), 16, 1024);
      const uint64_t sb_d = smem_desc(smem_u32(sm + L::kSb), 16384, 1024);
      const uint64_t es_d = smem_desc(smem_u32(sm + L::kEs), 8192, 1024);
      const uint64_t ed_d = smem_desc(smem_u32(sm + L::kEd), 8192, 1024);
      const uint64_t st_k = smem_desc(smem_u32(sm), 16, 1024);      // K-major tiles
      const uint64_t st_mn = smem_desc(smem_u32(sm), 8192, 1024);   // MN-major tiles
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % kTcStages;
        const uint32_t so = s * L::kStage;
        const uint32_t d1 = t_d1(c);
        if (!mbar_wait(&bars->full[s], (c / kTcStages) & 1, err, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk)  // D1 = [I ; 0] U
          mma_f16_ss(d1, desc_advance(id_d, kk * 32),
                     desc_advance(st_mn, so + L::kUQ + kk * 2048), id_kmn, kk > 0);
        if (!mbar_wait(&bars->s_ready, c & 1, err, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)  // D1 += [-Wk ; Q] Sb
          mma_f16_ss(d1, desc_advance(st_k, so + L::kA1 + (kk >> 2) * 16384 + (kk & 3) * 32),
                     desc_advance(sb_d, kk * 2048), id_kmn, 1);
        mma_commit(&bars->d1_full);
        if (!mbar_wait(&bars->e_ready, c & 1, err, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk)  // S += K^T Ed
          mma_f16_ss(t_s, desc_advance(st_mn, so + L::kK + kk * 2048),
                     desc_advance(ed_d, kk * 2048), id_mnmn, 1);
        mma_commit(&bars->d3_full);
        if (!mbar_wait(&bars->es_ready, c & 1, err, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk)  // D2 = [U ; QKm] Es
          mma_f16_ss(t_d2(c), desc_advance(st_k, so + L::kUQ + kk * 32),
                     desc_advance(es_d, kk * 2048), id_kmn, kk > 0);
        mma_commit(&bars->d2_full);
        mma_commit(&bars->empty[s]);
      }
      // Every MMA issued completes before TMEM is freed.
      mma_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, err, abort_flag, true);
    }
  } else {
    // ------------------------------------------------------- math warps 0-7
    const int q = warp & 3;                 // TMEM lane quadrant
    const int r = q * 32 + lane;            // accumulator row (state row / token row)
    const int cb = (warp >> 2) * 32;        // first column of this warp's half
    const int l = r & 63;                   // token of rows 0-63 / 64-127
    const bool err_rows = q < 2;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    uint8_t* Sb = sm + L::kSb;
    uint8_t* Es = sm + L::kEs;
    uint8_t* Ed = sm + L::kEd;
    bool ok = true;
    // This thread's 32 state values (fp32, row r, columns cb..cb+31) -> Sb in
    // bf16, then s_ready: MMA1 of the next chunk needs only Sb.
    auto publish_sb = [&](const uint32_t (&x)[32]) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint4 pk;
        pk.x = pack_bf16(__uint_as_float(x[8 * u + 0]), __uint_as_float(x[8 * u + 1]));
        pk.y = pack_bf16(__uint_as_float(x[8 * u + 2]), __uint_as_float(x[8 * u + 3]));
        pk.z = pack_bf16(__uint_as_float(x[8 * u + 4]), __uint_as_float(x[8 * u + 5]));
        pk.w = pack_bf16(__uint_as_float(x[8 * u + 6]), __uint_as_float(x[8 * u + 7]));
        *reinterpret_cast<uint4*>(Sb + swz(r, cb + 8 * u)) = pk;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->s_ready);
    };
    // Then, off the chain, the same values scaled by e^gc_last of chunk `next`
    // back to TMEM: MMA3 of chunk `next` accumulates onto them, and the issuer
    // starts it only after this thread's next e_ready arrival.
    auto prescale = [&](uint32_t (&x)[32], int next) {
      const int s = next % kTcStages;
      if (!mbar_wait(&bars->full[s], (next / kTcStages) & 1, err, abort_flag)) {
        ok = false;
        return;
      }
      const float egl = reinterpret_cast<const float*>(sm + L::kTail + s * L::kTailBytes)[2 * kC];
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = __float_as_uint(__uint_as_float(x[i]) * egl);
      tmem_st32(t_s + lane_off + cb, x);
      tmem_wait_st();
    };
    {
      uint32_t x[32];
#pragma unroll
      for (int i = 0; i < 32; ++i)
        x[i] = __float_as_uint(
            h0 ? h0[((static_cast<int64_t>(b) * H + h) * DK + r) * DV + v0 + cb + i] : 0.0f);
      publish_sb(x);
      prescale(x, 0);
    }
    for (int c = 0; ok && c < nchunks; ++c) {
      const int s = c % kTcStages;
      const float* tail = reinterpret_cast<const float*>(sm + L::kTail + s * L::kTailBytes);
      const int t0 = bos + c * kC;
      const int nvalid = min(kC, eos - t0);
      const int zpad = kVar ? nvalid : kC;  // padding rows to zero
      float qsc = 0.0f;
      if (err_rows) {
        // err = U - Wk S for token l (D1 rows 0-63) -> Es, Ed rows l.
        if (!mbar_wait(&bars->d1_full, c & 1, err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t x[32];
        tmem_ld32(t_d1(c) + lane_off + cb, x);
        tmem_wait_ld_regs(x);
        const float dec = tail[kC + l];
        // Ed (the decayed err, for MMA3 on the chain) first, then Es (MMA2).
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 pd;
          uint32_t* pdw = reinterpret_cast<uint32_t*>(&pd);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            pdw[e] = pack_bf16(dec * __uint_as_float(x[8 * u + 2 * e]),
                               dec * __uint_as_float(x[8 * u + 2 * e + 1]));
          *reinterpret_cast<uint4*>(Ed + swz(l, cb + 8 * u)) = pd;
        }
        if (l >= zpad) {
          // A padding row of packed sequences: its K row (box cb / 32 of the K tile) -> 0 before
          // MMA3 reads it (this thread waited for the stage in `prescale`).
          uint4* krow = reinterpret_cast<uint4*>(sm + s * L::kStage + L::kK + (cb >> 5) * 8192 +
                                                 l * 128);
#pragma unroll
          for (int u = 0; u < 8; ++u) krow[u] = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars->e_ready);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 pe;
          uint32_t* pew = reinterpret_cast<uint32_t*>(&pe);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            pew[e] = pack_bf16(__uint_as_float(x[8 * u + 2 * e]),
                               __uint_as_float(x[8 * u + 2 * e + 1]));
          *reinterpret_cast<uint4*>(Es + swz(l, cb + 8 * u)) = pe;
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->es_ready);
      } else {
        // Read before e_ready: the stage is refilled after MMA2, which the
        // issuer starts only after e_ready.  This arrival also orders this
        // thread's TMEM store of the pre-scaled state before MMA3.
        qsc = tail[l];
        tc_fence_before();
        mbar_arrive(&bars->e_ready);
      }
      // The new state: to Sb (bf16) and, pre-scaled for the next chunk, to TMEM.
      if (!mbar_wait(&bars->d3_full, c & 1, err, abort_flag)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t x[32];
        tmem_ld32(t_s + lane_off + cb, x);
        tmem_wait_ld_regs(x);
        if (c + 1 < nchunks) {
          publish_sb(x);
          prescale(x, c + 1);
        } else if (hT) {
          float* hrow = hT + ((static_cast<int64_t>(b) * H + h) * DK + r) * DV + v0 + cb;
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(hrow + i) =
                make_float4(__uint_as_float(x[i]), __uint_as_float(x[i + 1]),
                            __uint_as_float(x[i + 2]), __uint_as_float(x[i + 3]));
        }
      }
      if (!ok) break;
      if (!err_rows) {
        // o (token l) = qsc (Q S)[l] + (QKm err)[l], columns cb..cb+31.
        if (!mbar_wait(&bars->d2_full, c & 1, err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t x[32], y[32];
        tmem_ld32(t_d1(c) + lane_off + cb, x);
        tmem_ld32(t_d2(c) + lane_off + cb, y);
        tmem_wait_ld_regs(x);
        tmem_wait_ld_regs(y);
        if (l < nvalid) {
          uint4* orow = reinterpret_cast<uint4*>(
              o + (static_cast<int64_t>(t0 + l) * H + h) * DV + v0 + cb);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 pk;
            uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 8 * u + 2 * e;
              pw[e] = pack_bf16(fmaf(qsc, __uint_as_float(x[i]), __uint_as_float(y[i])),
                                fmaf(qsc, __uint_as_float(x[i + 1]), __uint_as_float(y[i + 1])));
            }
            orow[u] = pk;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kScanTcCols);
  }
}

// nseq sequences; `sl` says where they lie.  The q / k / v maps are (D, H,
// map_rows, map_batch): (T, B) for a uniform batch, (total, 1) for packed
// sequences.  For variable length, sl.chunk_seq points at nslots ints the
// index kernel fills first.
template <int DK, int DV, bool kVar, bool kNorm>
int launch_gdn(const void* q, const void* k, const void* v, const float* g, const float* beta,
               const float* h0, void* o, float* hT, void* ws, SeqLayout sl, int nseq,
               int map_rows, int map_batch, int H, float scale, cudaStream_t s) {
  auto k1 = gdn_prepare<DK, DV, kVar, kNorm>;
  auto k2 = gdn_scan<DK, DV, kVar>;
  CUtensorMap tq, tk, tv;
  if (!make_bshd_map(&tq, q, DK, H, map_rows, map_batch, kC, true) ||
      !make_bshd_map(&tk, k, DK, H, map_rows, map_batch, kC, true) ||
      !make_bshd_map(&tv, v, DV, H, map_rows, map_batch, kC, true))
    return TILEOPS_ELAUNCH;
  const int smem1 = PrepSmem<DK, DV>::kAlloc;
  const int smem2 = ScanSmem<DK>::kAlloc;
  // Workspace tiles as 3-D maps (columns, 64 rows, chunk units).
  const uint64_t units = static_cast<uint64_t>(H) * sl.nslots;
  const uint64_t wb = Ws<DK, DV>::kBytes;
  CUtensorMap twk, tu, tqk;
  {
    auto* base = static_cast<const uint8_t*>(ws);
    const uint64_t dk_dims[3] = {DK, kC, units}, dk_str[2] = {DK * 2, wb};
    const uint64_t dv_dims[3] = {DV, kC, units}, dv_str[2] = {DV * 2, wb};
    const uint64_t c_dims[3] = {kC, kC, units}, c_str[2] = {kC * 2, wb};
    const uint32_t box[3] = {64, kC, 1};
    if (!make_tiled_map_16bit(&twk, base + Ws<DK, DV>::kWk * 2, true, 3, dk_dims, dk_str, box) ||
        !make_tiled_map_16bit(&tu, base + Ws<DK, DV>::kU * 2, true, 3, dv_dims, dv_str, box) ||
        !make_tiled_map_16bit(&tqk, base + Ws<DK, DV>::kQK * 2, true, 3, c_dims, c_str, box))
      return TILEOPS_ELAUNCH;
  }
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1) !=
          cudaSuccess ||
      cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2) != cudaSuccess)
    return TILEOPS_ELAUNCH;
  if (units > 0x7fffffffULL) return TILEOPS_EBADSHAPE;
  if constexpr (kVar) {
    gdn_chunk_index<<<(sl.nslots + 255) / 256, 256, 0, s>>>(sl, nseq,
                                                            const_cast<int*>(sl.chunk_seq),
                                                            device_error_ptr());
    const int st = launch_status();
    if (st != TILEOPS_OK) return st;
  }
  k1<<<static_cast<unsigned>(units), 128, smem1, s>>>(
      tq, tk, tv, twk, tu, g, beta, static_cast<__nv_bfloat16*>(ws), sl, H, scale,
      device_error_ptr());
  int st = launch_status();
  if (st != TILEOPS_OK) return st;
  const unsigned grid2 = static_cast<unsigned>(nseq * H * (DV / kSlice));
  if constexpr (DK == 128) {
    // dk = 128: the tensor-core (tcgen05) scan; its final-state stores are
    // 16-byte vectors, so it needs an aligned final_state.
    if (hT == nullptr || aligned16(hT)) {
      auto k3 = gdn_scan_tc<DV, kVar>;
      if (cudaFuncSetAttribute(k3, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               ScanTcSmem::kAlloc) != cudaSuccess)
        return TILEOPS_ELAUNCH;
      k3<<<grid2, kScanTcThreads, ScanTcSmem::kAlloc, s>>>(
          tq, tk, twk, tu, tqk, static_cast<const __nv_bfloat16*>(ws), h0,
          static_cast<__nv_bfloat16*>(o), hT, sl, H, device_error_ptr());
      return launch_status();
    }
  }
  k2<<<grid2, 256, smem2, s>>>(tq, tk, twk, tu, tqk, static_cast<const __nv_bfloat16*>(ws), h0,
                               static_cast<__nv_bfloat16*>(o), hT, sl, H, device_error_ptr());
  return launch_status();
}

int64_t ws_bytes_per_chunk(int64_t dim_k, int64_t dim_v) {
  if (dim_k == 128 && dim_v == 128) return Ws<128, 128>::kBytes;
  if (dim_k == 64 && dim_v == 64) return Ws<64, 64>::kBytes;
  if (dim_k == 128 && dim_v == 64) return Ws<128, 64>::kBytes;
  if (dim_k == 64 && dim_v == 128) return Ws<64, 128>::kBytes;
  return -1;
}

// Variable length: chunk slots per head, and where the chunk -> sequence
// table sits in the workspace (after the chunk units, 16-byte aligned).
int64_t varlen_slots(int64_t total_len, int64_t num_seqs) { return total_len / kC + num_seqs; }
int64_t varlen_table_offset(int64_t total_len, int64_t num_seqs, int64_t heads, int64_t per) {
  return heads * varlen_slots(total_len, num_seqs) * per;
}

template <bool kVar, bool kNorm>
int dispatch_gdn(const void* q, const void* k, const void* v, const float* g, const float* beta,
                 const float* h0, void* o, float* hT, void* ws, SeqLayout sl, int nseq,
                 int map_rows, int map_batch, int H, int dim_k, int dim_v, float scale,
                 cudaStream_t s) {
  if (dim_k == 128 && dim_v == 128)
    return launch_gdn<128, 128, kVar, kNorm>(q, k, v, g, beta, h0, o, hT, ws, sl, nseq, map_rows, map_batch,
                                H, scale, s);
  if (dim_k == 64 && dim_v == 64)
    return launch_gdn<64, 64, kVar, kNorm>(q, k, v, g, beta, h0, o, hT, ws, sl, nseq, map_rows, map_batch, H,
                              scale, s);
  if (dim_k == 128 && dim_v == 64)
    return launch_gdn<128, 64, kVar, kNorm>(q, k, v, g, beta, h0, o, hT, ws, sl, nseq, map_rows, map_batch,
                               H, scale, s);
  return launch_gdn<64, 128, kVar, kNorm>(q, k, v, g, beta, h0, o, hT, ws, sl, nseq, map_rows, map_batch, H,
                             scale, s);
}

}  // namespace
}  // namespace tileops

using namespace tileops;

extern "C" int64_t tileops_gdn_workspace_bytes(int64_t batch, int64_t seq_len, int64_t heads,
                                               int64_t dim_k, int64_t dim_v) {
  if (batch < 0 || seq_len < 0 || heads <= 0) return -1;
  const int64_t nchunks = (seq_len + kC - 1) / kC;
  const int64_t per = ws_bytes_per_chunk(dim_k, dim_v);
  if (per < 0) return -1;
  return batch * heads * nchunks * per;
}

extern "C" int tileops_gdn_prefill_fwd(const void* q, const void* k, const void* v,
                                       const float* g, const float* beta,
                                       const float* initial_state, void* o,
                                       float* final_state, void* workspace, int64_t batch,
                                       int64_t seq_len, int64_t heads, int64_t dim_k,
                                       int64_t dim_v, int64_t chunk_size, double scale,
                                       int dtype, void* stream) {
  if (batch < 0 || seq_len < 0 || heads <= 0 || batch * heads > (1 << 24) ||
      seq_len > (1 << 30) || batch * seq_len > 0x7fffffffLL)
    return TILEOPS_EBADSHAPE;
  if (chunk_size != kC) return TILEOPS_EBADSHAPE;
  if (ws_bytes_per_chunk(dim_k, dim_v) < 0) return TILEOPS_EBADSHAPE;
  if (dtype != TILEOPS_DT_BF16) return TILEOPS_EBADDTYPE;
  if (batch == 0 || seq_len == 0) return TILEOPS_OK;
  if (!q || !k || !v || !g || !beta || !o || !workspace) return TILEOPS_EINVAL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(workspace))
    return TILEOPS_EALIGN;
  const int B = static_cast<int>(batch), T = static_cast<int>(seq_len);
  const int nchunks = (T + kC - 1) / kC;
  const SeqLayout sl{nullptr, nullptr, T, nchunks, B * nchunks};
  return dispatch_gdn<false, false>(q, k, v, g, beta, initial_state, o, final_state, workspace,
                                    sl, B, T, B,
                      static_cast<int>(heads), static_cast<int>(dim_k), static_cast<int>(dim_v),
                      static_cast<float>(scale), as_stream(stream));
}

extern "C" int64_t tileops_gdn_varlen_workspace_bytes(int64_t total_len, int64_t num_seqs,
                                                      int64_t heads, int64_t dim_k,
                                                      int64_t dim_v) {
  if (total_len < 0 || num_seqs < 0 || heads <= 0) return -1;
  const int64_t per = ws_bytes_per_chunk(dim_k, dim_v);
  if (per < 0) return -1;
  const int64_t table = (varlen_slots(total_len, num_seqs) * 4 + 15) / 16 * 16;
  return varlen_table_offset(total_len, num_seqs, heads, per) + table;
}

extern "C" int tileops_gdn_prefill_varlen_fwd(const void* q, const void* k, const void* v,
                                              const float* g, const float* beta,
                                              const int32_t* cu_seqlens, int64_t num_seqs,
                                              const float* initial_state, void* o,
                                              float* final_state, void* workspace,
                                              int64_t total_len, int64_t heads, int64_t dim_k,
                                              int64_t dim_v, int64_t chunk_size, double scale,
                                              int flags, int dtype, void* stream) {
  if (total_len < 0 || num_seqs < 0 || heads <= 0 || total_len > (1 << 30) ||
      num_seqs > (1 << 24) || heads * varlen_slots(total_len, num_seqs) > 0x7fffffffLL ||
      num_seqs * heads > (1 << 24))
    return TILEOPS_EBADSHAPE;
  if (chunk_size != kC) return TILEOPS_EBADSHAPE;
  const int64_t per = ws_bytes_per_chunk(dim_k, dim_v);
  if (per < 0) return TILEOPS_EBADSHAPE;
  if (dtype != TILEOPS_DT_BF16) return TILEOPS_EBADDTYPE;
  if ((flags & ~TILEOPS_GDN_QK_L2NORM) != 0) return TILEOPS_EINVAL;
  if (cu_seqlens == nullptr && num_seqs > 0 && total_len % num_seqs != 0)
    return TILEOPS_EBADSHAPE;
  if (num_seqs == 0) return TILEOPS_OK;
  cudaStream_t s = as_stream(stream);
  const int64_t state_bytes = num_seqs * heads * dim_k * dim_v * 4;
  if (total_len == 0) {  // every sequence is empty: final state = initial state
    if (!final_state) return TILEOPS_OK;
    const cudaError_t e =
        initial_state ? cudaMemcpyAsync(final_state, initial_state, state_bytes,
                                        cudaMemcpyDeviceToDevice, s)
                      : cudaMemsetAsync(final_state, 0, state_bytes, s);
    return e == cudaSuccess ? TILEOPS_OK : TILEOPS_ELAUNCH;
  }
  if (!q || !k || !v || !g || !beta || !o || !workspace) return TILEOPS_EINVAL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(workspace))
    return TILEOPS_EALIGN;
  const bool norm = (flags & TILEOPS_GDN_QK_L2NORM) != 0;
  const int H = static_cast<int>(heads), N = static_cast<int>(num_seqs);
  const int dk = static_cast<int>(dim_k), dv = static_cast<int>(dim_v);
  const float sc = static_cast<float>(scale);
  if (cu_seqlens == nullptr) {  // num_seqs sequences of total_len / num_seqs rows each
    const int T = static_cast<int>(total_len / num_seqs);
    const int nchunks = (T + kC - 1) / kC;
    const SeqLayout sl{nullptr, nullptr, T, nchunks, N * nchunks};
    return norm ? dispatch_gdn<false, true>(q, k, v, g, beta, initial_state, o, final_state,
                                            workspace, sl, N, T, N, H, dk, dv, sc, s)
                : dispatch_gdn<false, false>(q, k, v, g, beta, initial_state, o, final_state,
                                             workspace, sl, N, T, N, H, dk, dv, sc, s);
  }
  const int64_t nslots = varlen_slots(total_len, num_seqs);
  auto* table = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                       varlen_table_offset(total_len, num_seqs, heads, per));
  const SeqLayout sl{cu_seqlens, table, static_cast<int>(total_len), 0,
                     static_cast<int>(nslots)};
  const int rows = static_cast<int>(total_len);
  return norm ? dispatch_gdn<true, true>(q, k, v, g, beta, initial_state, o, final_state,
                                         workspace, sl, N, rows, 1, H, dk, dv, sc, s)
              : dispatch_gdn<true, false>(q, k, v, g, beta, initial_state, o, final_state,
                                          workspace, sl, N, rows, 1, H, dk, dv, sc, s);
}

// ------------------------------------------------------------------------
// No-allocation variant.
//
// Some callers cannot allocate device memory at call time: code running
// inside a captured CUDA graph or an allocator-free runtime (a C host that
// never links the CUDA allocator, a plugin that owns no memory pool, a
// signal-safe or real-time path where cudaMalloc may block or fail).  For
// them this entry point runs the same two kernels with the per-chunk WY
// factors kept in a fixed scratch array that lives in the library's own
// device memory instead of a caller-provided workspace.
//
// Limits and contract:
//  * The scratch is kGdnStaticScratchBytes (16 MiB) per GPU, held by every GPU
//    that loads this library until the process exits.  A shape needs
//    tileops_gdn_workspace_bytes(...) bytes of it (41,488 bytes per 64-token
//    chunk of every (batch, head) at dk = dv = 128, so at most 404 such
//    chunks, e.g. batch * heads = 16 with seq_len <= 1,600); larger shapes are
//    rejected with TILEOPS_EBADSHAPE before anything is enqueued.
//  * All calls share the one array: two calls whose kernels overlap on the GPU
//    (different streams, or different host threads) race on it.
//  * Nothing in the scratch has to start at zero: the prepare kernel writes
//    every byte the scan kernel reads for the chunks in use.
//  * The first call on each device (with that device current) looks up the
//    device addresses of both library symbols a GDN call uses -- this array
//    and the device error word that the kernels' bounded waits write -- with
//    cudaGetSymbolAddress, which may load the module lazily; make that first
//    call outside any stream capture.  Later calls only read the cached
//    addresses (one entry per device index, any index).
constexpr size_t kGdnStaticScratchBytes = static_cast<size_t>(16) << 20;
static __device__ __align__(256) unsigned char g_gdn_static_scratch[kGdnStaticScratchBytes];

namespace {
void* gdn_static_scratch_ptr() {
  static std::mutex mu;
  static std::vector<void*> cached;  // by device index
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cached.size() <= static_cast<size_t>(dev)) cached.resize(static_cast<size_t>(dev) + 1, nullptr);
  if (!cached[dev]) {
    // Resolve the error word too, so one first call covers every lookup.
    if (!tileops::device_error_ptr()) return nullptr;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gdn_static_scratch) != cudaSuccess) return nullptr;
    cached[dev] = p;
  }
  return cached[dev];
}
}  // namespace

extern "C" int tileops_gdn_prefill_fwd_noalloc(const void* q, const void* k, const void* v,
                                               const float* g, const float* beta,
                                               const float* initial_state, void* o,
                                               float* final_state, int64_t batch,
                                               int64_t seq_len, int64_t heads, int64_t dim_k,
                                               int64_t dim_v, int64_t chunk_size, double scale,
                                               int dtype, void* stream) {
  const int64_t need = tileops_gdn_workspace_bytes(batch, seq_len, heads, dim_k, dim_v);
  if (need < 0) return TILEOPS_EBADSHAPE;
  if (static_cast<uint64_t>(need) > kGdnStaticScratchBytes) return TILEOPS_EBADSHAPE;
  if (batch == 0 || seq_len == 0) return TILEOPS_OK;
  void* scratch = gdn_static_scratch_ptr();
  if (!scratch) return TILEOPS_ELAUNCH;
  return tileops_gdn_prefill_fwd(q, k, v, g, beta, initial_state, o, final_state, scratch,
                                 batch, seq_len, heads, dim_k, dim_v, chunk_size, scale, dtype,
                                 stream);
}
