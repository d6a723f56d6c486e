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
// Kernel 1 (gdn_prepare): one CTA per (b, h, chunk).  KK^T and QK^T on tensor
// cores (mma.sync bf16, fp32 accumulate); T by 16 x 16 block forward
// substitution in fp32 (diagonal blocks by substitution, off-diagonal blocks
// by T_ij = -T_ii sum_m A_im T_mj); Wk and U as tensor-core products with T.
// Results go to a caller-provided workspace, 64 x (dk + dv + 64) bf16 plus 64
// fp32 per chunk.
// Kernel 2 (gdn_scan): one CTA per (b, h, 64-wide slice of dv) -- the columns
// of S evolve independently -- walking the chunks in order.  S lives in fp32
// registers as MMA accumulators; every chunk's operands are prefetched one
// chunk ahead with cp.async into padded (bank-conflict free) shared memory.
//
// Layout: q, k (B, T, H, dk) bf16; v, o (B, T, H, dv) bf16; g, beta (B, T, H)
// fp32; initial / final state (B, H, dk, dv) fp32.  Tokens past T are
// treated as k = v = q = 0, g = beta = 0 (they leave the state unchanged).
#include <mutex>

#include "common.cuh"

namespace tileops {
namespace {

constexpr int kC = 64;  // chunk length

// ---------------------------------------------------- warp-level MMA helpers
__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr(p)));
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

// A fragment (16 x 16) of a row-major [m][k] bf16 tile, rows m0.., cols k0..
__device__ __forceinline__ void frag_a(uint32_t (&a)[4], const __nv_bfloat16* base, int ld,
                                       int m0, int k0) {
  const int lane = threadIdx.x & 31;
  ldsm_x4(a, base + (m0 + (lane & 15)) * ld + k0 + ((lane >> 4) << 3));
}
// A fragment of A = X^T where X is stored row-major [k][m].
__device__ __forceinline__ void frag_a_t(uint32_t (&a)[4], const __nv_bfloat16* base, int ld,
                                         int m0, int k0) {
  const int lane = threadIdx.x & 31;
  const int mat = lane >> 3;  // 0: (m0,k0) 1: (m0+8,k0) 2: (m0,k0+8) 3: (m0+8,k0+8)
  ldsm_x4_t(a, base + (k0 + (lane & 7) + ((mat >> 1) << 3)) * ld + m0 + ((mat & 1) << 3));
}
// B fragments of two adjacent n-tiles (n0.., n0+8..) where B[k][n] is stored
// row-major [k][n]: b[0..1] for tile n0, b[2..3] for tile n0 + 8.
__device__ __forceinline__ void frag_b_kn(uint32_t (&b)[4], const __nv_bfloat16* base, int ld,
                                          int k0, int n0) {
  const int lane = threadIdx.x & 31;
  const int mat = lane >> 3;  // 0: (k0,n0) 1: (k0+8,n0) 2: (k0,n0+8) 3: (k0+8,n0+8)
  ldsm_x4_t(b, base + (k0 + (lane & 7) + ((mat & 1) << 3)) * ld + n0 + ((mat >> 1) << 3));
}
// B fragments of two adjacent n-tiles where B[k][n] = X[n][k], X row-major [n][k].
__device__ __forceinline__ void frag_b_nk(uint32_t (&b)[4], const __nv_bfloat16* base, int ld,
                                          int k0, int n0) {
  const int lane = threadIdx.x & 31;
  const int mat = lane >> 3;  // 0: (n0,k0) 1: (n0,k0+8) 2: (n0+8,k0) 3: (n0+8,k0+8)
  ldsm_x4(b, base + (n0 + (lane & 7) + ((mat >> 1) << 3)) * ld + k0 + ((mat & 1) << 3));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool valid) {
  // src-size 0 writes 16 zero bytes (out-of-range token).
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Workspace of one chunk (element offsets into a bf16 array, then fp32 tail).
template <int DK, int DV>
struct Ws {
  static constexpr int64_t kWk = 0;                 // C x DK bf16
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

// =========================================================== kernel 1
// 128 threads.  Shared memory (bf16 tiles padded by 8 columns):
//   Ks [64][DK+8] (later overwritten in place by Kp = beta e^gc K),
//   Qs [64][DK+8] (later reused for Ts, T in bf16 [64][72]),
//   Vs [64][DV+8] (later overwritten in place by Vp = beta V),
//   As, Tf: fp32 [64][65]; gc, beta: [64].
template <int DK, int DV>
struct PrepSmem {
  static constexpr int kLdK = DK + 8, kLdV = DV + 8, kLdT = kC + 8, kLdF = kC + 1;
  static constexpr int kKs = 0;
  static constexpr int kQs = kKs + kC * kLdK * 2;
  static constexpr int kVs = kQs + kC * kLdK * 2;
  static constexpr int kAs = kVs + kC * kLdV * 2;
  static constexpr int kTf = kAs + kC * kLdF * 4;
  static constexpr int kGc = kTf + kC * kLdF * 4;
  static constexpr int kBeta = kGc + kC * 4;
  static constexpr int kBytes = kBeta + kC * 4;
};

template <int DK, int DV>
__global__ void __launch_bounds__(128)
    gdn_prepare(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
                const float* __restrict__ beta, __nv_bfloat16* __restrict__ ws, int T, int H,
                int nchunks, float scale) {
  using L = PrepSmem<DK, DV>;
  using W = Ws<DK, DV>;
  extern __shared__ __align__(16) uint8_t sm[];
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(sm + L::kKs);
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(sm + L::kQs);
  __nv_bfloat16* Vs = reinterpret_cast<__nv_bfloat16*>(sm + L::kVs);
  __nv_bfloat16* Kp = Ks;  // in place, once KK^T is done
  __nv_bfloat16* Vp = Vs;
  __nv_bfloat16* Ts = Qs;  // once QK^T is done
  float* As = reinterpret_cast<float*>(sm + L::kAs);
  float* Tf = reinterpret_cast<float*>(sm + L::kTf);
  float* gc = reinterpret_cast<float*>(sm + L::kGc);
  float* bt = reinterpret_cast<float*>(sm + L::kBeta);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = blockIdx.x % nchunks;
  const int bh = blockIdx.x / nchunks;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int t0 = chunk * kC;
  __nv_bfloat16* wsc = ws + static_cast<int64_t>(blockIdx.x) * (W::kBytes / 2);
  float* wsf = reinterpret_cast<float*>(wsc);

  // ---- load K, Q, V rows of the chunk (zero past T) and g, beta
  {
    constexpr int kPkK = DK / 8, kPkV = DV / 8;  // 16-byte packets per row
    for (int i = tid; i < kC * kPkK; i += 128) {
      const int r = i / kPkK, c = (i - r * kPkK) * 8;
      const int t = t0 + r;
      const bool ok = t < T;
      const int64_t off = ((static_cast<int64_t>(b) * T + (ok ? t : 0)) * H + h) * DK + c;
      cp_async16_zfill(Ks + r * L::kLdK + c, k + off, ok);
      cp_async16_zfill(Qs + r * L::kLdK + c, q + off, ok);
    }
    for (int i = tid; i < kC * kPkV; i += 128) {
      const int r = i / kPkV, c = (i - r * kPkV) * 8;
      const int t = t0 + r;
      const bool ok = t < T;
      const int64_t off = ((static_cast<int64_t>(b) * T + (ok ? t : 0)) * H + h) * DV + c;
      cp_async16_zfill(Vs + r * L::kLdV + c, v + off, ok);
    }
    cp_commit();
  }
  if (warp == 0) {
    // inclusive cumsum of g over the 64 tokens: two per lane + warp scan
    float g0 = 0.0f, g1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
    const int ta = t0 + 2 * lane, tb = ta + 1;
    if (ta < T) {
      const int64_t o = (static_cast<int64_t>(b) * T + ta) * H + h;
      g0 = g[o];
      b0 = beta[o];
    }
    if (tb < T) {
      const int64_t o = (static_cast<int64_t>(b) * T + tb) * H + h;
      g1 = g[o];
      b1 = beta[o];
    }
    float pair = g0 + g1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float up = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += up;
    }
    const float excl = incl - pair;
    gc[2 * lane] = excl + g0;
    gc[2 * lane + 1] = incl;
    bt[2 * lane] = b0;
    bt[2 * lane + 1] = b1;
  }
  cp_wait<0>();
  __syncthreads();

  // ---- KK^T -> A (strictly lower, fp32) and QK^T -> QKm (bf16, to workspace)
  {
    const int m0 = warp * 16;
    const int g8 = lane >> 2, t2 = (lane & 3) * 2;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const __nv_bfloat16* X = which == 0 ? Ks : Qs;
      float acc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < DK / 16; ++kk) {
        uint32_t a[4];
        frag_a(a, X, L::kLdK, m0, kk * 16);
#pragma unroll
        for (int n = 0; n < 8; n += 2) {
          uint32_t bb[4];
          frag_b_nk(bb, Ks, L::kLdK, kk * 16, n * 8);
          mma_bf16(acc[n], a, bb[0], bb[1]);
          mma_bf16(acc[n + 1], a, bb[2], bb[3]);
        }
      }
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int l = m0 + g8 + ((e >> 1) << 3), s = n * 8 + t2 + (e & 1);
          const float dec = __expf(gc[l] - gc[s]);
          if (which == 0) {
            As[l * L::kLdF + s] = l > s ? bt[l] * dec * acc[n][e] : 0.0f;
          } else {
            wsc[W::kQK + l * kC + s] = __float2bfloat16_rn(l >= s ? scale * dec * acc[n][e] : 0.0f);
          }
        }
    }
  }
  __syncthreads();

  // ---- in place: Kp = beta e^gc K, Vp = beta V; the fp32 tail of the workspace
  {
    const float gl = gc[kC - 1];
    for (int i = tid; i < kC * DK; i += 128) {
      const int r = i / DK, c = i - r * DK;
      Kp[r * L::kLdK + c] =
          __float2bfloat16_rn(bt[r] * __expf(gc[r]) * __bfloat162float(Ks[r * L::kLdK + c]));
    }
    for (int i = tid; i < kC * DV; i += 128) {
      const int r = i / DV, c = i - r * DV;
      Vp[r * L::kLdV + c] = __float2bfloat16_rn(bt[r] * __bfloat162float(Vs[r * L::kLdV + c]));
    }
    if (tid < kC) {
      wsf[W::kQsc + tid] = scale * __expf(gc[tid]);
      wsf[W::kDec + tid] = __expf(gl - gc[tid]);
    }
    if (tid < 4) wsf[W::kEgl + tid] = tid == 0 ? __expf(gl) : 0.0f;
  }

  // ---- T = (I + A)^-1, 16 x 16 blocks, fp32
  // (1) diagonal blocks by forward substitution: thread (blk, col) owns one column.
  if (tid < kC) {
    const int blk = tid >> 4, col = tid & 15, base = blk * 16;
    float t[16];
#pragma unroll
    for (int l = 0; l < 16; ++l) {
      float acc = 0.0f;
#pragma unroll
      for (int m = 0; m < l; ++m) acc = fmaf(As[(base + l) * L::kLdF + base + m], t[m], acc);
      t[l] = (l == col) ? 1.0f : (l > col ? -acc : 0.0f);
    }
#pragma unroll
    for (int l = 0; l < 16; ++l) Tf[(base + l) * L::kLdF + base + col] = t[l];
  }
  // zero the strictly upper blocks
  for (int i = tid; i < kC * kC; i += 128) {
    const int r = i >> 6, c = i & 63;
    if ((c >> 4) > (r >> 4)) Tf[r * L::kLdF + c] = 0.0f;
  }
  __syncthreads();
  // (2) off-diagonal blocks, by distance d = i - j = 1, 2, 3:
  //     T_ij = -T_ii (sum_{m=j}^{i-1} A_im T_mj); 16 x 16 x 16 products on CUDA cores.
  for (int d = 1; d < 4; ++d) {
    const int nblocks = 4 - d;  // pairs (i, j = i - d)
    // step a: X_ij = sum_m A_im T_mj  -> stored in As block (i, j) (A_ij no longer needed)
    for (int e = tid; e < nblocks * 256; e += 128) {
      const int pidx = e >> 8, rc = e & 255, r = rc >> 4, c = rc & 15;
      const int i = pidx + d, j = pidx;
      float acc = 0.0f;
      for (int m = j; m < i; ++m)
#pragma unroll
        for (int x = 0; x < 16; ++x)
          acc = fmaf(As[(i * 16 + r) * L::kLdF + m * 16 + x], Tf[(m * 16 + x) * L::kLdF + j * 16 + c],
                     acc);
      Tf[(i * 16 + r) * L::kLdF + j * 16 + c] = acc;  // temporarily X_ij
    }
    __syncthreads();
    // step b: T_ij = -T_ii X_ij (read X from Tf, write result back after a barrier)
    float res[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // (4 - d) * 256 / 128 <= 6 per thread
    int cnt = 0;
    for (int e = tid; e < nblocks * 256; e += 128, ++cnt) {
      const int pidx = e >> 8, rc = e & 255, r = rc >> 4, c = rc & 15;
      const int i = pidx + d, j = pidx;
      float acc = 0.0f;
#pragma unroll
      for (int x = 0; x < 16; ++x)
        acc = fmaf(Tf[(i * 16 + r) * L::kLdF + i * 16 + x], Tf[(i * 16 + x) * L::kLdF + j * 16 + c],
                   acc);
      res[cnt] = -acc;
    }
    __syncthreads();
    cnt = 0;
    for (int e = tid; e < nblocks * 256; e += 128, ++cnt) {
      const int pidx = e >> 8, rc = e & 255, r = rc >> 4, c = rc & 15;
      const int i = pidx + d, j = pidx;
      Tf[(i * 16 + r) * L::kLdF + j * 16 + c] = res[cnt];
    }
    __syncthreads();
  }
  for (int i = tid; i < kC * kC; i += 128) {
    const int r = i >> 6, c = i & 63;
    Ts[r * L::kLdT + c] = __float2bfloat16_rn(Tf[r * L::kLdF + c]);
  }
  __syncthreads();

  // ---- Wk = T Kp (C x DK), U = T Vp (C x DV): warp w owns rows 16w..16w+15
  {
    const int m0 = warp * 16;
    const int g8 = lane >> 2, t2 = (lane & 3) * 2;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const int D = which == 0 ? DK : DV;
      const int ld = which == 0 ? L::kLdK : L::kLdV;
      const __nv_bfloat16* X = which == 0 ? Kp : Vp;
      __nv_bfloat16* out = wsc + (which == 0 ? W::kWk : W::kU);
      for (int n0 = 0; n0 < D; n0 += 64) {
        float acc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
        for (int kk = 0; kk <= warp; ++kk) {  // T is lower triangular
          uint32_t a[4];
          frag_a(a, Ts, L::kLdT, m0, kk * 16);
#pragma unroll
          for (int n = 0; n < 8; n += 2) {
            uint32_t bb[4];
            frag_b_kn(bb, X, ld, kk * 16, n0 + n * 8);
            mma_bf16(acc[n], a, bb[0], bb[1]);
            mma_bf16(acc[n + 1], a, bb[2], bb[3]);
          }
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int l = m0 + g8, c = n0 + n * 8 + t2;
          *reinterpret_cast<uint32_t*>(out + l * D + c) = pack_bf16(acc[n][0], acc[n][1]);
          *reinterpret_cast<uint32_t*>(out + (l + 8) * D + c) = pack_bf16(acc[n][2], acc[n][3]);
        }
      }
    }
  }
}

// =========================================================== kernel 2
// 256 threads (8 warps), one CTA per (b, h, 64-column slice of dv).
// Per-stage shared memory (padded bf16): Qs, Ks, Wks [64][DK+8];
// Us [64][72] (the slice); QKs [64][72]; eg [64] + gl.  Two stages.
// Plus Ss [DK][72] (S in bf16, B operand), Es / Ed [64][72] (err and
// decayed err, B operands).
constexpr int kSlice = 64;

template <int DK>
struct ScanSmem {
  static constexpr int kLdK = DK + 8, kLdS = kSlice + 8;
  static constexpr int kQs = 0;
  static constexpr int kKs = kQs + kC * kLdK * 2;
  static constexpr int kWks = kKs + kC * kLdK * 2;
  static constexpr int kUs = kWks + kC * kLdK * 2;
  static constexpr int kQKs = kUs + kC * kLdS * 2;
  static constexpr int kEg = kQKs + kC * kLdS * 2;  // the workspace fp32 tail
  static constexpr int kStage = kEg + (2 * kC + 4) * 4;
  static constexpr int kSs = 2 * kStage;
  static constexpr int kEs = kSs + DK * kLdS * 2;
  static constexpr int kEd = kEs + kC * kLdS * 2;
  static constexpr int kBytes = kEd + kC * kLdS * 2;
};

template <int DK, int DV>
__global__ void __launch_bounds__(256, 1)
    gdn_scan(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
             const __nv_bfloat16* __restrict__ ws, const float* __restrict__ h0,
             __nv_bfloat16* __restrict__ o, float* __restrict__ hT, int T, int H,
             int nchunks) {
  using L = ScanSmem<DK>;
  using W = Ws<DK, DV>;
  extern __shared__ __align__(16) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kSlices = DV / kSlice;
  const int slice = blockIdx.x % kSlices;
  const int bh = blockIdx.x / kSlices;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int v0 = slice * kSlice;
  const int g8 = lane >> 2, t2 = (lane & 3) * 2;

  auto stage_ptr = [&](int s, int off) { return sm + s * L::kStage + off; };
  auto prefetch = [&](int s, int chunk) {
    const int t0 = chunk * kC;
    const __nv_bfloat16* wsc = ws + (static_cast<int64_t>(bh) * nchunks + chunk) * (W::kBytes / 2);
    __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(stage_ptr(s, L::kQs));
    __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(stage_ptr(s, L::kKs));
    __nv_bfloat16* Wks = reinterpret_cast<__nv_bfloat16*>(stage_ptr(s, L::kWks));
    __nv_bfloat16* Us = reinterpret_cast<__nv_bfloat16*>(stage_ptr(s, L::kUs));
    __nv_bfloat16* QKs = reinterpret_cast<__nv_bfloat16*>(stage_ptr(s, L::kQKs));
    float* egs = reinterpret_cast<float*>(stage_ptr(s, L::kEg));
    constexpr int kPkK = DK / 8;
    for (int i = tid; i < kC * kPkK; i += 256) {
      const int r = i / kPkK, c = (i - r * kPkK) * 8;
      const int t = t0 + r;
      const bool ok = t < T;
      const int64_t off = ((static_cast<int64_t>(b) * T + (ok ? t : 0)) * H + h) * DK + c;
      cp_async16_zfill(Qs + r * L::kLdK + c, q + off, ok);
      cp_async16_zfill(Ks + r * L::kLdK + c, k + off, ok);
      cp_async16(Wks + r * L::kLdK + c, wsc + W::kWk + r * DK + c);
    }
    for (int i = tid; i < kC * (kSlice / 8); i += 256) {
      const int r = i >> 3, c = (i & 7) * 8;
      cp_async16(Us + r * L::kLdS + c, wsc + W::kU + r * DV + v0 + c);
      cp_async16(QKs + r * L::kLdS + c, wsc + W::kQK + r * kC + c);
    }
    if (tid < W::kTailFloats / 4)
      cp_async16(egs + tid * 4, reinterpret_cast<const float*>(wsc) + W::kQsc + tid * 4);
  };

  __nv_bfloat16* Ss = reinterpret_cast<__nv_bfloat16*>(sm + L::kSs);
  __nv_bfloat16* Es = reinterpret_cast<__nv_bfloat16*>(sm + L::kEs);
  __nv_bfloat16* Ed = reinterpret_cast<__nv_bfloat16*>(sm + L::kEd);

  prefetch(0, 0);
  cp_commit();

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

  for (int chunk = 0; chunk < nchunks; ++chunk) {
    const int s = chunk & 1;
    if (chunk + 1 < nchunks) prefetch(s ^ 1, chunk + 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();  // chunk's data and the published state are visible
    const __nv_bfloat16* Qs = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(s, L::kQs));
    const __nv_bfloat16* Ks = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(s, L::kKs));
    const __nv_bfloat16* Wks = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(s, L::kWks));
    const __nv_bfloat16* Us = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(s, L::kUs));
    const __nv_bfloat16* QKs = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(s, L::kQKs));
    const float* egs = reinterpret_cast<const float*>(stage_ptr(s, L::kEg));
    const float* qsc = egs;            // scale * exp(gc_l)
    const float* dcy = egs + kC;       // exp(gc_last - gc_l)
    const float egl = egs[2 * kC];     // exp(gc_last)
    // err = U - Wk S ; qs = Q S   (this warp's 16 x 32 tile)
    float ws_acc[4][4], qs_acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) ws_acc[n][e] = qs_acc[n][e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
      uint32_t aw[4], aq[4];
      frag_a(aw, Wks, L::kLdK, om0, kk * 16);
      frag_a(aq, Qs, L::kLdK, om0, kk * 16);
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
        const __nv_bfloat162 u2 = *reinterpret_cast<const __nv_bfloat162*>(Us + l * L::kLdS + c);
        const float e0 = __bfloat162float(u2.x) - ws_acc[n][half * 2];
        const float e1 = __bfloat162float(u2.y) - ws_acc[n][half * 2 + 1];
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
      frag_a(a, QKs, L::kLdS, om0, kk * 16);
#pragma unroll
      for (int n = 0; n < 4; n += 2) {
        uint32_t bb[4];
        frag_b_kn(bb, Es, L::kLdS, kk * 16, on0 + n * 8);
        mma_bf16(o_acc[n], a, bb[0], bb[1]);
        mma_bf16(o_acc[n + 1], a, bb[2], bb[3]);
      }
    }
    {
      const int t0 = chunk * kC;
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int l = om0 + g8 + half * 8, c = on0 + n * 8 + t2;
          const int t = t0 + l;
          if (t < T)
            *reinterpret_cast<uint32_t*>(o + ((static_cast<int64_t>(b) * T + t) * H + h) * DV +
                                         v0 + c) = pack_bf16(o_acc[n][half * 2],
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
        frag_a_t(a, Ks, L::kLdK, sr0, kk * 16);
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
  cp_wait<0>();
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

template <int DK, int DV>
int launch_gdn(const void* q, const void* k, const void* v, const float* g, const float* beta,
               const float* h0, void* o, float* hT, void* ws, int B, int T, int H, float scale,
               cudaStream_t s) {
  const int nchunks = (T + kC - 1) / kC;
  auto k1 = gdn_prepare<DK, DV>;
  auto k2 = gdn_scan<DK, DV>;
  const int smem1 = PrepSmem<DK, DV>::kBytes;
  const int smem2 = ScanSmem<DK>::kBytes;
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1) !=
          cudaSuccess ||
      cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2) != cudaSuccess)
    return TILEOPS_ELAUNCH;
  const int64_t grid1 = static_cast<int64_t>(B) * H * nchunks;
  if (grid1 > 0x7fffffffLL) return TILEOPS_EBADSHAPE;
  k1<<<static_cast<unsigned>(grid1), 128, smem1, s>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(v), g, beta, static_cast<__nv_bfloat16*>(ws), T, H,
      nchunks, scale);
  int st = launch_status();
  if (st != TILEOPS_OK) return st;
  k2<<<static_cast<unsigned>(B * H * (DV / kSlice)), 256, smem2, s>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(ws), h0, static_cast<__nv_bfloat16*>(o), hT, T, H,
      nchunks);
  return launch_status();
}

}  // namespace
}  // namespace tileops

using namespace tileops;

extern "C" int64_t tileops_gdn_workspace_bytes(int64_t batch, int64_t seq_len, int64_t heads,
                                               int64_t dim_k, int64_t dim_v) {
  if (batch < 0 || seq_len < 0 || heads <= 0) return -1;
  const int64_t nchunks = (seq_len + kC - 1) / kC;
  int64_t per = 0;
  if (dim_k == 128 && dim_v == 128) per = Ws<128, 128>::kBytes;
  else if (dim_k == 64 && dim_v == 64) per = Ws<64, 64>::kBytes;
  else if (dim_k == 128 && dim_v == 64) per = Ws<128, 64>::kBytes;
  else if (dim_k == 64 && dim_v == 128) per = Ws<64, 128>::kBytes;
  else return -1;
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
      seq_len > (1 << 30))
    return TILEOPS_EBADSHAPE;
  if (chunk_size != kC) return TILEOPS_EBADSHAPE;
  if (!((dim_k == 64 || dim_k == 128) && (dim_v == 64 || dim_v == 128))) return TILEOPS_EBADSHAPE;
  if (dtype != TILEOPS_DT_BF16) return TILEOPS_EBADDTYPE;
  if (batch == 0 || seq_len == 0) return TILEOPS_OK;
  if (!q || !k || !v || !g || !beta || !o || !workspace) return TILEOPS_EINVAL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(workspace))
    return TILEOPS_EALIGN;
  cudaStream_t s = as_stream(stream);
  const int B = static_cast<int>(batch), T = static_cast<int>(seq_len), H = static_cast<int>(heads);
  const float sc = static_cast<float>(scale);
  if (dim_k == 128 && dim_v == 128)
    return launch_gdn<128, 128>(q, k, v, g, beta, initial_state, o, final_state, workspace, B, T,
                                H, sc, s);
  if (dim_k == 64 && dim_v == 64)
    return launch_gdn<64, 64>(q, k, v, g, beta, initial_state, o, final_state, workspace, B, T, H,
                              sc, s);
  if (dim_k == 128 && dim_v == 64)
    return launch_gdn<128, 64>(q, k, v, g, beta, initial_state, o, final_state, workspace, B, T,
                               H, sc, s);
  return launch_gdn<64, 128>(q, k, v, g, beta, initial_state, o, final_state, workspace, B, T, H,
                             sc, s);
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
//  * The device address of the array is looked up (cudaGetSymbolAddress) on
//    the first call on each device, with that device current; make that first
//    call outside any stream capture.
constexpr size_t kGdnStaticScratchBytes = static_cast<size_t>(16) << 20;
static __device__ __align__(256) unsigned char g_gdn_static_scratch[kGdnStaticScratchBytes];

namespace {
void* gdn_static_scratch_ptr() {
  static std::mutex mu;
  static void* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[dev]) {
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
