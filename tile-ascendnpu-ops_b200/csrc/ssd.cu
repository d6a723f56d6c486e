// Mamba-2 State-Space Dual (SSD) chunk scan, forward: the output of every
// chunk from its incoming state and its own tokens.
//
// Per batch b, chunk c, head h (group g = h / (H / G)), rows l of the chunk:
//   out[l, p] = exp(dA[l]) * sum_n C[l, n] prev[p, n]                 (history)
//             + sum_{s <= l} cb[l, s] exp(dA[l] - dA[s]) dt[s] x[s, p]   (intra)
// Layouts (mamba_ssm _chunk_scan_fwd): x (B, S, H, P) and C (B, S, G, N) in
// the 16-bit dtype, S = NC Q; cb (B, NC, G, Q, Q) dtype; dA_cumsum (B, H, NC,
// Q) fp32; prev_states (B, NC, H, P, N) fp32; dt (B, H, NC, Q) dtype; out
// (B, S, H, P) fp32.
// Reference: SSDChunkScanFwdOp, examples/TileOPs/tileops/ops/mamba/ssd_chunk_scan.py:29
// and kernels/mamba/ssd_chunk_scan/ssd_chunk_scan_kernel/perf_opt/
// _ssd_chunk_scan_fwd_kernel.py:181 (golden at :123-178).
//
// One CTA (128 threads) per (b, c, h, 128-row tile of the chunk); thread r
// owns row l0 + r (TMEM lane r).  Both terms are tcgen05 MMAs (M = 128,
// N = P, kind::f16, fp32 accumulators in TMEM):
//   D1 = C_tile [128 x N] . prev^T        A K-major (C rows), B K-major (prev
//                                          rows p, converted fp32 -> dtype)
//   D2 = W [128 x s] . x [s x P]          A = W built per 64-key block in
//                                          registers, B MN-major (x rows s)
// with W[l, s] = cb[l, s] exp(dA[l] - dA[s]) dt[s] for s <= l (< Q), else 0.
// Operands are staged with cp.async (16-byte copies, zero fill past the
// chunk / past N) into 128-byte-swizzled shared tiles; the W and x blocks are
// double-buffered so block j+1 is built while the tensor core runs block j.
// Epilogue: out = exp(dA[l]) D1 + D2 straight from TMEM to global fp32.
// Every mbarrier wait is bounded (2 s); a timeout sets the device error flag,
// the MMAs issued so far are drained and TMEM is freed before returning.
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace tileops {
namespace {

using namespace sm100;

constexpr int kSsdThreads = 128;
constexpr int kSsdRows = 128;   // chunk rows per CTA (MMA M)
constexpr int kSsdKBlk = 64;    // keys per W / x block
constexpr int kSsdMaxN = 256;   // d_state
constexpr int kSsdMaxP = 128;   // d_head
constexpr int kSsdMaxQ = 1024;  // chunk length

// 16-byte unit u of 128-byte row r of a swizzled 64-column tile.
__device__ __forceinline__ uint32_t ssd_swz(int r, int u) {
  return static_cast<uint32_t>(r * 128 + ((u ^ (r & 7)) << 4));
}

struct SsdSmem {
  static constexpr int kC = 0;                                     // [128][256] K-major
  static constexpr int kPrev = kC + kSsdRows * kSsdMaxN * 2;       // [P][256] K-major
  static constexpr int kW = kPrev + kSsdMaxP * kSsdMaxN * 2;       // 2 x [128][64]
  static constexpr int kX = kW + 2 * kSsdRows * kSsdKBlk * 2;      // 2 x [64][128] MN-major
  static constexpr int kDA = kX + 2 * kSsdKBlk * kSsdMaxP * 2;     // Q floats
  static constexpr int kDt = kDA + kSsdMaxQ * 4;                   // Q floats
  static constexpr int kBar = kDt + kSsdMaxQ * 4;                  // mbarriers, tmem base
  static constexpr int kBytes = kBar + 64;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 232448, "SSD shared memory exceeds 227 KB");
};

struct SsdBars {
  uint64_t blk_done[2];  // MMAs of the W / x block in buffer i completed
  uint64_t all_done;     // every MMA completed
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack16(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack16<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack16<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

struct SsdParams {
  const void* x;
  const void* cb;
  const float* dA;
  const void* C;
  const float* prev;
  const void* dt;
  float* out;
  int B, NC, Q, H, P, N, G;
  int ltiles;  // ceil(Q / 128)
  int* err;
};

template <typename T>
__global__ void __launch_bounds__(kSsdThreads, 1) ssd_chunk_scan(const SsdParams p) {
  using L = SsdSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  SsdBars* bars = reinterpret_cast<SsdBars*>(sm + L::kBar);
  volatile int* abort_flag = &bars->abort_flag;
  float* sdA = reinterpret_cast<float*>(sm + L::kDA);
  float* sdt = reinterpret_cast<float*>(sm + L::kDt);
  const uint32_t sb = smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5;

  // CTA -> (b, c, h, row tile); consecutive CTAs share (b, c): cb and C rows
  // are read by every head of the group from L2.
  int bx = blockIdx.x;
  const int lt = bx % p.ltiles;
  bx /= p.ltiles;
  const int h = bx % p.H;
  const int bc = bx / p.H;  // b * NC + c
  const int b = bc / p.NC, c = bc - b * p.NC;
  const int g = h / (p.H / p.G);
  const int Q = p.Q, P = p.P, N = p.N;
  const int l0 = lt * kSsdRows;
  const int S = p.NC * Q;
  const int npad = (N + 15) & ~15;                 // K of the history MMA
  const int kend = min(Q, l0 + kSsdRows);          // keys s < kend matter
  const int nblk = (kend + kSsdKBlk - 1) / kSsdKBlk;

  if (tid == 0) {
    mbar_init(&bars->blk_done[0], 1);
    mbar_init(&bars->blk_done[1], 1);
    mbar_init(&bars->all_done, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, 256);
    tmem_relinquish();
  }

  // ---- per-chunk scalars: dA (fp32) and dt -> shared
  const int64_t hc = (static_cast<int64_t>(b) * p.H + h) * p.NC + c;
  for (int i = tid; i < Q; i += kSsdThreads) {
    sdA[i] = p.dA[hc * Q + i];
    sdt[i] = Cvt<T>::to_f(static_cast<const T*>(p.dt)[hc * Q + i]);
  }

  // ---- C tile (rows l0.., n < npad) by cp.async, zero past the chunk / N
  {
    const T* Cg = static_cast<const T*>(p.C);
    const int upr = npad / 8;  // 16-byte units per row
    for (int i = tid; i < kSsdRows * upr; i += kSsdThreads) {
      const int r = i / upr, u = i - r * upr;
      const int l = l0 + r, n = u * 8;
      const bool ok = l < Q && n < N;
      const T* src = Cg + ((static_cast<int64_t>(b) * S + c * Q + (ok ? l : 0)) * p.G + g) * N +
                     (ok ? n : 0);
      cp_async16(sb + L::kC + (n >> 6) * (kSsdRows * 128) + ssd_swz(r, (n & 63) >> 3), src, ok);
    }
  }
  // ---- prev (P x N fp32) -> dtype, K-major [p][n]
  {
    const float* pg = p.prev + ((static_cast<int64_t>(b) * p.NC + c) * p.H + h) * P * N;
    const int upr = npad / 8;
    for (int i = tid; i < P * upr; i += kSsdThreads) {
      const int r = i / upr, u = i - r * upr, n = u * 8;
      uint4 pk = make_uint4(0u, 0u, 0u, 0u);
      if (n < N) {
        const float4 a = *reinterpret_cast<const float4*>(pg + static_cast<int64_t>(r) * N + n);
        const float4 d = *reinterpret_cast<const float4*>(pg + static_cast<int64_t>(r) * N + n + 4);
        pk.x = pack16<T>(a.x, a.y);
        pk.y = pack16<T>(a.z, a.w);
        pk.z = pack16<T>(d.x, d.y);
        pk.w = pack16<T>(d.z, d.w);
      }
      *reinterpret_cast<uint4*>(sm + L::kPrev + (n >> 6) * (P * 128) + ssd_swz(r, (n & 63) >> 3)) =
          pk;
    }
  }
  __syncthreads();  // sdA / sdt visible

  // W and x of key block j into buffer j & 1.
  const T* xg = static_cast<const T*>(p.x);
  const T* cbg = static_cast<const T*>(p.cb) +
                 ((static_cast<int64_t>(b) * p.NC + c) * p.G + g) * static_cast<int64_t>(Q) * Q;
  auto stage = [&](int j) {
    const int buf = j & 1;
    const int s0 = j * kSsdKBlk;
    // x rows s0.. (MN-major, P columns in 64-wide chunks)
    const int upr = P / 8;
    for (int i = tid; i < kSsdKBlk * upr; i += kSsdThreads) {
      const int r = i / upr, u = i - r * upr;
      const int s = s0 + r, pc = u * 8;
      const bool ok = s < Q;
      const T* src = xg + ((static_cast<int64_t>(b) * S + c * Q + (ok ? s : 0)) * p.H + h) * P + pc;
      cp_async16(sb + L::kX + buf * (kSsdKBlk * kSsdMaxP * 2) + (pc >> 6) * (kSsdKBlk * 128) +
                     ssd_swz(r, (pc & 63) >> 3),
                 src, ok);
    }
    // W rows (thread: packet column tid & 7 = keys s0 + 8 (tid & 7).., rows tid >> 3 + 16 i)
    const int cp = tid & 7, rg = tid >> 3;
    const int sc = s0 + cp * 8;
    float das[8], dts[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int s = sc + e;
      das[e] = s < Q ? sdA[s] : 0.0f;
      dts[e] = s < Q ? sdt[s] : 0.0f;
    }
    const bool vec = (Q & 7) == 0;
#pragma unroll 2
    for (int it = 0; it < kSsdRows / 16; ++it) {
      const int r = rg + 16 * it;
      const int l = l0 + r;
      float w[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) w[e] = 0.0f;
      if (l < Q && sc <= l) {
        T cv[8];
        const T* row = cbg + static_cast<int64_t>(l) * Q + sc;
        if (vec && sc + 8 <= Q) {
          *reinterpret_cast<uint4*>(cv) = *reinterpret_cast<const uint4*>(row);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) cv[e] = sc + e < Q ? row[e] : Cvt<T>::from_f(0.0f);
        }
        const float dal = sdA[l];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (sc + e <= l) w[e] = Cvt<T>::to_f(cv[e]) * __expf(dal - das[e]) * dts[e];
      }
      uint4 pk;
      pk.x = pack16<T>(w[0], w[1]);
      pk.y = pack16<T>(w[2], w[3]);
      pk.z = pack16<T>(w[4], w[5]);
      pk.w = pack16<T>(w[6], w[7]);
      *reinterpret_cast<uint4*>(sm + L::kW + buf * (kSsdRows * 128) + ssd_swz(r, cp)) = pk;
    }
  };

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t id_kk = idesc_f16_major(kSsdRows, P, kBf16 ? 1 : 0, 0, 0);
  const uint32_t id_kmn = idesc_f16_major(kSsdRows, P, kBf16 ? 1 : 0, 0, 1);
  stage(0);
  cp_async_wait_all();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t t_d1 = tmem, t_d2 = tmem + 128;
  bool ok = true;
  int issued = 0;  // key blocks whose MMAs were issued
  for (int j = 0; j < nblk; ++j) {
    const int buf = j & 1;
    if (j > 0) {
      // Buffer `buf` was last read by block j - 2's MMAs.
      if (j >= 2 && !mbar_wait(&bars->blk_done[buf], ((j - 2) >> 1) & 1, p.err, abort_flag)) {
        ok = false;
      }
      if (!__syncthreads_and(ok)) {
        ok = false;
        break;
      }
      stage(j);
      cp_async_wait_all();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
    }
    if (tid == 0) {
      if (j == 0) {
        const uint64_t a = smem_desc(sb + L::kC, 16, 1024);
        const uint64_t bd = smem_desc(sb + L::kPrev, 16, 1024);
        for (int kk = 0; kk < npad / 16; ++kk)
          mma_f16_ss(t_d1, desc_advance(a, (kk >> 2) * (kSsdRows * 128) + (kk & 3) * 32),
                     desc_advance(bd, (kk >> 2) * (P * 128) + (kk & 3) * 32), id_kk, kk > 0);
      }
      const uint64_t a = smem_desc(sb + L::kW + buf * (kSsdRows * 128), 16, 1024);
      const uint64_t bd =
          smem_desc(sb + L::kX + buf * (kSsdKBlk * kSsdMaxP * 2), kSsdKBlk * 128, 1024);
#pragma unroll
      for (int kk = 0; kk < kSsdKBlk / 16; ++kk)
        mma_f16_ss(t_d2, desc_advance(a, kk * 32), desc_advance(bd, kk * 16 * 128), id_kmn,
                   (j > 0 || kk > 0) ? 1u : 0u);
      mma_commit(&bars->blk_done[buf]);
    }
    issued = j + 1;
  }
  if (tid == 0) mma_commit(&bars->all_done);
  // All threads wait for the accumulators (with a failed run: for the MMAs
  // already issued, so TMEM is not freed under them).
  const bool done = mbar_wait(&bars->all_done, 0, p.err, abort_flag, !ok);
  tc_fence_after();
  if (ok && done && issued == nblk) {
    const int r = tid;
    const int l = l0 + r;
    const uint32_t lane = static_cast<uint32_t>(warp * 32) << 16;
    const float eh = l < Q ? __expf(sdA[l]) : 0.0f;
    float* orow = p.out + ((static_cast<int64_t>(b) * S + c * Q + l) * p.H + h) * P;
    for (int c0 = 0; c0 < P; c0 += 32) {
      uint32_t x1[32], x2[32];
      tmem_ld32(t_d1 + lane + c0, x1);
      tmem_ld32(t_d2 + lane + c0, x2);
      tmem_wait_ld_regs(x1);
      tmem_wait_ld_regs(x2);
      if (l < Q) {
        const int ncol = min(32, P - c0);
        for (int i = 0; i < ncol; i += 4)
          *reinterpret_cast<float4*>(orow + c0 + i) =
              make_float4(fmaf(eh, __uint_as_float(x1[i]), __uint_as_float(x2[i])),
                          fmaf(eh, __uint_as_float(x1[i + 1]), __uint_as_float(x2[i + 1])),
                          fmaf(eh, __uint_as_float(x1[i + 2]), __uint_as_float(x2[i + 2])),
                          fmaf(eh, __uint_as_float(x1[i + 3]), __uint_as_float(x2[i + 3])));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

template <typename T>
int launch_ssd(const SsdParams& p, cudaStream_t s) {
  auto k = ssd_chunk_scan<T>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SsdSmem::kAlloc) !=
      cudaSuccess)
    return TILEOPS_ELAUNCH;
  const int64_t grid = static_cast<int64_t>(p.B) * p.NC * p.H * p.ltiles;
  k<<<static_cast<unsigned>(grid), kSsdThreads, SsdSmem::kAlloc, s>>>(p);
  return launch_status();
}

}  // namespace
}  // namespace tileops

using namespace tileops;

extern "C" int tileops_ssd_chunk_scan_fwd(const void* x, const void* cb, const float* dA_cumsum,
                                          const void* C, const float* prev_states,
                                          const void* dt, float* out, int64_t batch,
                                          int64_t num_chunks, int64_t chunk_len, int64_t n_heads,
                                          int64_t d_head, int64_t d_state, int64_t n_groups,
                                          int dtype, void* stream) {
  if (batch < 0 || num_chunks < 0 || chunk_len <= 0 || n_heads <= 0 || n_groups <= 0 ||
      n_heads % n_groups != 0)
    return TILEOPS_EBADSHAPE;
  if (d_head <= 0 || d_head > kSsdMaxP || d_head % 16 != 0) return TILEOPS_EBADSHAPE;
  if (d_state <= 0 || d_state > kSsdMaxN || d_state % 8 != 0) return TILEOPS_EBADSHAPE;
  if (chunk_len > kSsdMaxQ) return TILEOPS_EBADSHAPE;
  if (dtype != TILEOPS_DT_BF16 && dtype != TILEOPS_DT_F16) return TILEOPS_EBADDTYPE;
  const int64_t ltiles = (chunk_len + kSsdRows - 1) / kSsdRows;
  const int64_t grid = batch * num_chunks * n_heads * ltiles;
  if (grid > 0x7fffffffLL || batch * num_chunks * chunk_len > 0x7fffffffLL)
    return TILEOPS_EBADSHAPE;
  if (grid == 0) return TILEOPS_OK;
  if (!x || !cb || !dA_cumsum || !C || !prev_states || !dt || !out) return TILEOPS_EINVAL;
  if (!aligned16(x) || !aligned16(C) || !aligned16(prev_states) || !aligned16(out) ||
      !aligned16(cb))
    return TILEOPS_EALIGN;
  SsdParams p;
  p.x = x;
  p.cb = cb;
  p.dA = dA_cumsum;
  p.C = C;
  p.prev = prev_states;
  p.dt = dt;
  p.out = out;
  p.B = static_cast<int>(batch);
  p.NC = static_cast<int>(num_chunks);
  p.Q = static_cast<int>(chunk_len);
  p.H = static_cast<int>(n_heads);
  p.P = static_cast<int>(d_head);
  p.N = static_cast<int>(d_state);
  p.G = static_cast<int>(n_groups);
  p.ltiles = static_cast<int>(ltiles);
  p.err = device_error_ptr();
  cudaStream_t s = as_stream(stream);
  return dtype == TILEOPS_DT_BF16 ? launch_ssd<__nv_bfloat16>(p, s) : launch_ssd<__half>(p, s);
}
