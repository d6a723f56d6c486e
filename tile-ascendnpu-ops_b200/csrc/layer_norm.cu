// Fused residual add + LayerNorm forward.
//
//   s   = round_T(x + residual)                      -> residual_out
//   y   = round_T((s - mean(s)) * rstd * w + b)      -> y
//   rstd = 1 / sqrt(mean((s - mean)^2) + eps)
//
// The statistics are taken over the ROUNDED sum s (what the reference's
// ref_program normalises: tests/ops/test_fused_add_layer_norm.py:55-72 and
// golden_fused_add_layer_norm in
// kernels/norm/fused_add_layer_norm/fused_add_layer_norm_kernel/_fused_add_layer_norm_kernel.py:118-134),
// two-pass (mean, then centred variance) in fp32 like the reference kernel
// (_fused_add_layer_norm_fwd_kernels.py:79-94).
//
// Design: one CTA per row.  Each thread owns VPT 16-byte packets of the row
// (packet j of thread t is column packet t + j*blockDim), keeps s in fp32
// registers between the two reductions and the output pass, so x and
// residual are read exactly once and y / residual_out written once: the
// kernel moves the algorithmic (4*M*N)*sizeof(T) + 2*N*sizeof(W) bytes.
// Reductions are warp shuffles plus one shared-memory exchange across warps.
// Rows too wide for registers (more than 4 packets per thread at 1024
// threads) use a three-pass kernel that re-reads residual_out from L2.
//
// Many rows of 1K..8K elements (the hot configuration, 8192 x 4096 bf16):
// a persistent kernel with a per-thread cp.async prefetch ring, see
// faln_ring below.
#include "common.cuh"

namespace tileops {
namespace {

template <typename T, int V>
struct RowPack {
  // V elements of T starting at an element offset.  V == 16/sizeof(T) uses
  // one 16-byte access; V == 1 is the scalar path for ragged / misaligned rows.
  T e[V];
  __device__ __forceinline__ void load_stream(const T* p) {
    if constexpr (V * sizeof(T) == 16) {
      uint4 u = ld_stream(p);
      memcpy(e, &u, 16);
    } else {
      for (int i = 0; i < V; ++i) e[i] = p[i];
    }
  }
  __device__ __forceinline__ void store_stream(T* p) const {
    if constexpr (V * sizeof(T) == 16) {
      uint4 u;
      memcpy(&u, e, 16);
      st_stream(p, u);
    } else {
      for (int i = 0; i < V; ++i) p[i] = e[i];
    }
  }
};

// Load V affine parameters (reused by every row: normal cached loads).
template <typename W, int V>
__device__ __forceinline__ void load_affine(const W* __restrict__ p, float* out, bool vec) {
  if (vec) {
    constexpr int kBytes = V * sizeof(W);
    static_assert(kBytes % 16 == 0 || kBytes < 16, "affine packet");
    if constexpr (kBytes >= 16) {
      W tmp[V];
#pragma unroll
      for (int q = 0; q < kBytes / 16; ++q) {
        uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + q);
        memcpy(reinterpret_cast<char*>(tmp) + 16 * q, &u, 16);
      }
#pragma unroll
      for (int i = 0; i < V; ++i) out[i] = Cvt<W>::to_f(tmp[i]);
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) out[i] = Cvt<W>::to_f(p[i]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the CTA; every thread gets the total.  `red` holds 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();  // `red` may still be read by the previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? red[lane] : 0.0f;
  return warp_sum(t);
}

template <typename T, typename W, int V, int VPT>
__global__ void __launch_bounds__(1024)
    faln_rows(const T* __restrict__ x, const T* __restrict__ res, const W* __restrict__ w,
              const W* __restrict__ b, T* __restrict__ y, T* __restrict__ res_out, int64_t N,
              float eps, bool affine_vec) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t npk = N / V;  // caller guarantees N % V == 0
  const T* xr = x + row * N;
  const T* rr = res + row * N;
  T* yr = y + row * N;
  T* sr = res_out + row * N;

  float s[VPT][V];
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t p = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
    if (p < npk) {
      RowPack<T, V> a, c;
      a.load_stream(xr + p * V);
      c.load_stream(rr + p * V);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        a.e[i] = Cvt<T>::from_f(Cvt<T>::to_f(a.e[i]) + Cvt<T>::to_f(c.e[i]));
        s[j][i] = Cvt<T>::to_f(a.e[i]);
        sum += s[j][i];
      }
      a.store_stream(sr + p * V);
    } else {
#pragma unroll
      for (int i = 0; i < V; ++i) s[j][i] = 0.0f;
    }
  }
  const float inv_n = 1.0f / static_cast<float>(N);
  const float mean = block_sum(sum, red) * inv_n;
  float sq = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t p = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
    if (p < npk) {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float d = s[j][i] - mean;
        sq += d * d;
      }
    }
  }
  const float var = block_sum(sq, red) * inv_n;
  const float rstd = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t p = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
    if (p < npk) {
      float wv[V], bv[V];
      load_affine<W, V>(w + p * V, wv, affine_vec);
      load_affine<W, V>(b + p * V, bv, affine_vec);
      RowPack<T, V> o;
#pragma unroll
      for (int i = 0; i < V; ++i) o.e[i] = Cvt<T>::from_f((s[j][i] - mean) * rstd * wv[i] + bv[i]);
      o.store_stream(yr + p * V);
    }
  }
}

// Any N: three passes over the row, the later two re-reading the rounded sum
// from residual_out (L2-resident for the rows in flight).
template <typename T, typename W>
__global__ void __launch_bounds__(1024)
    faln_rows_wide(const T* __restrict__ x, const T* __restrict__ res, const W* __restrict__ w,
                   const W* __restrict__ b, T* __restrict__ y, T* __restrict__ res_out,
                   int64_t N, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * N;
  const T* rr = res + row * N;
  T* yr = y + row * N;
  T* sr = res_out + row * N;
  float sum = 0.0f;
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x) {
    const T sv = Cvt<T>::from_f(Cvt<T>::to_f(xr[c]) + Cvt<T>::to_f(rr[c]));
    sr[c] = sv;
    sum += Cvt<T>::to_f(sv);
  }
  const float inv_n = 1.0f / static_cast<float>(N);
  const float mean = block_sum(sum, red) * inv_n;
  float sq = 0.0f;
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x) {
    const float d = Cvt<T>::to_f(sr[c]) - mean;
    sq += d * d;
  }
  const float var = block_sum(sq, red) * inv_n;
  const float rstd = 1.0f / sqrtf(var + eps);
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x)
    yr[c] = Cvt<T>::from_f((Cvt<T>::to_f(sr[c]) - mean) * rstd * Cvt<W>::to_f(w[c]) +
                           Cvt<W>::to_f(b[c]));
}


// ------------------------------------------------- prefetch-ring path
// Persistent CTAs (as many as are resident), each walking rows blockIdx.x,
// +gridDim.x, ...  Every thread copies ITS OWN packets of the rows STAGES-1
// ahead into a private slot of a shared-memory ring with cp.async (16 bytes
// per instruction, L1 bypassed), so
//   * the loads of the next rows are in flight while the CTA reduces and
//     writes the current one (the row's HBM latency is hidden), and
//   * no barrier is needed for the staged data: a thread only ever reads
//     back what it copied (cp.async.wait_group orders it).
// The ring is laid out thread-major (slot q of thread t at q*256 + t), so
// both the copies and the reads are bank-conflict free.

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Sum over the CTA into every thread with ONE barrier: lane 0 of each warp
// publishes its warp's sum in `buf`, then every thread adds the published
// values.  Callers alternate two buffers, so a buffer is only rewritten after
// a barrier that every reader of its previous contents has passed.
__device__ __forceinline__ float block_sum_1bar(float v, float* buf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  if (lane == 0) buf[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int i = 0; i < nwarps; ++i) t += buf[i];
  return t;
}

template <typename T, typename W, int VPT, int kRingThreads, int kRingStages>
__global__ void __launch_bounds__(kRingThreads)
    faln_ring(const T* __restrict__ x, const T* __restrict__ res, const W* __restrict__ w,
              const W* __restrict__ b, T* __restrict__ y, T* __restrict__ res_out, int64_t M,
              int64_t N, float eps, bool affine_vec) {
  constexpr int V = 16 / sizeof(T);
  extern __shared__ uint4 ring[];  // [kRingStages][2 * VPT][kRingThreads]
  __shared__ float red[2][32];
  const int tid = threadIdx.x;
  const int64_t npk = N / V;
  const int64_t grid = gridDim.x;
  auto slot = [&](int stage, int q) -> uint4* {
    return ring + (static_cast<int64_t>(stage) * 2 * VPT + q) * kRingThreads + tid;
  };
  auto prefetch = [&](int stage, int64_t row) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t p = tid + static_cast<int64_t>(j) * kRingThreads;
      if (p < npk) {
        cp_async16(slot(stage, j), x + row * N + p * V);
        cp_async16(slot(stage, VPT + j), res + row * N + p * V);
      }
    }
  };
#pragma unroll
  for (int s = 0; s < kRingStages - 1; ++s) {
    const int64_t row = blockIdx.x + s * grid;
    if (row < M) prefetch(s, row);
    cp_async_commit();  // one group per row slot, empty past the end
  }
  // A thread owns the same columns in every row: its weight / bias stay in
  // registers for the whole kernel.
  float wv[VPT][V], bv[VPT][V];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t p = tid + static_cast<int64_t>(j) * kRingThreads;
    if (p < npk) {
      load_affine<W, V>(w + p * V, wv[j], affine_vec);
      load_affine<W, V>(b + p * V, bv[j], affine_vec);
    }
  }
  const float inv_n = 1.0f / static_cast<float>(N);
  int it = 0;
  for (int64_t row = blockIdx.x; row < M; row += grid, ++it) {
    {
      const int64_t ahead = row + (kRingStages - 1) * grid;
      // Slot (it-1) % STAGES: this thread finished reading it last iteration.
      if (ahead < M) prefetch((it + kRingStages - 1) % kRingStages, ahead);
      cp_async_commit();
    }
    cp_async_wait<kRingStages - 1>();  // the group of this row has landed
    const int stage = it % kRingStages;
    T* sr = res_out + row * N;
    float v[VPT][V];
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t p = tid + static_cast<int64_t>(j) * kRingThreads;
      if (p < npk) {
        Pack16<T> a, c;
        a.u = *slot(stage, j);
        c.u = *slot(stage, VPT + j);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          a.e[i] = Cvt<T>::from_f(Cvt<T>::to_f(a.e[i]) + Cvt<T>::to_f(c.e[i]));
          v[j][i] = Cvt<T>::to_f(a.e[i]);
          sum += v[j][i];
        }
        st_stream(sr + p * V, a.u);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) v[j][i] = 0.0f;
      }
    }
    const float mean = block_sum_1bar(sum, red[0]) * inv_n;
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t p = tid + static_cast<int64_t>(j) * kRingThreads;
      if (p < npk) {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const float d = v[j][i] - mean;
          sq += d * d;
        }
      }
    }
    const float rstd = 1.0f / sqrtf(block_sum_1bar(sq, red[1]) * inv_n + eps);
    T* yr = y + row * N;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t p = tid + static_cast<int64_t>(j) * kRingThreads;
      if (p < npk) {
        Pack16<T> o;
#pragma unroll
        for (int i = 0; i < V; ++i)
          o.e[i] = Cvt<T>::from_f((v[j][i] - mean) * rstd * wv[j][i] + bv[j][i]);
        st_stream(yr + p * V, o.u);
      }
    }
  }
  cp_async_wait<0>();  // no copy may land after the CTA exits
}

// Ring geometry for a row of npk packets: THREADS threads own VPT packets
// each; STAGES-1 rows are prefetched.  Returns false when no variant fits.
template <typename T, typename W, int VPT, int THREADS, int STAGES>
int launch_ring(const T* x, const T* r, const W* w, const W* b, T* y, T* so, int64_t M,
                int64_t N, float eps, bool affine_vec, cudaStream_t s) {
  auto kern = faln_ring<T, W, VPT, THREADS, STAGES>;
  const size_t smem = static_cast<size_t>(STAGES) * 2 * VPT * THREADS * 16;
  // The kernel's static shared memory counts against the same 48 KB default,
  // so the opt-in is always requested.
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return TILEOPS_ELAUNCH;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, THREADS, smem) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int64_t grid64 = static_cast<int64_t>(sm_count()) * per_sm;
  const unsigned grid = static_cast<unsigned>(grid64 < M ? grid64 : M);
  kern<<<grid, THREADS, smem, s>>>(x, r, w, b, y, so, M, N, eps, affine_vec);
  return launch_status();
}

template <typename T, typename W>
bool try_launch_ring(const T* x, const T* r, const W* w, const W* b, T* y, T* so, int64_t M,
                     int64_t N, float eps, bool affine_vec, cudaStream_t s, int* status) {
  constexpr int V = 16 / sizeof(T);
  const int64_t npk = N / V;
  // Rows of 128 .. 1024 packets (N = 1024 .. 8192 for 16-bit types) and
  // enough rows for several per CTA.
  if (npk < 128 || npk > 1024 || M < 4 * sm_count()) return false;
  // Depth: about 64 KB of rows in flight per CTA, two CTAs per SM (measured
  // on B200 for 8192 x 4096 bf16: 5 stages of 16 KB beat 3, 4, 6, 8 and 12,
  // and 256 threads x 2 packets beat 128 x 4 and 512 x 1).
  if (npk <= 256)
    *status = launch_ring<T, W, 2, 128, 8>(x, r, w, b, y, so, M, N, eps, affine_vec, s);
  else if (npk <= 512)
    *status = launch_ring<T, W, 2, 256, 5>(x, r, w, b, y, so, M, N, eps, affine_vec, s);
  else
    *status = launch_ring<T, W, 4, 256, 3>(x, r, w, b, y, so, M, N, eps, affine_vec, s);
  return true;
}

template <typename T, typename W, int V>
int launch_rows(const T* x, const T* r, const W* w, const W* b, T* y, T* so, int64_t M,
                int64_t N, float eps, bool affine_vec, cudaStream_t s) {
  const int64_t npk = N / V;
  // 256 threads unless the row needs more than 4 packets per thread (the
  // register budget of a 1024-thread CTA is 64 per thread: 4 packets of 8
  // fp32 values fit, 8 would spill).
  int threads = 256;
  if (npk < 256) threads = static_cast<int>(((npk + 31) / 32) * 32);
  while (threads < 1024 && (npk + threads - 1) / threads > 4) threads *= 2;
  const int64_t vpt = (npk + threads - 1) / threads;
  const unsigned grid = static_cast<unsigned>(M);
  if (vpt <= 1)
    faln_rows<T, W, V, 1><<<grid, threads, 0, s>>>(x, r, w, b, y, so, N, eps, affine_vec);
  else if (vpt <= 2)
    faln_rows<T, W, V, 2><<<grid, threads, 0, s>>>(x, r, w, b, y, so, N, eps, affine_vec);
  else if (vpt <= 4)
    faln_rows<T, W, V, 4><<<grid, threads, 0, s>>>(x, r, w, b, y, so, N, eps, affine_vec);
  else
    faln_rows_wide<T, W><<<grid, 1024, 0, s>>>(x, r, w, b, y, so, N, eps);
  return launch_status();
}

template <typename T, typename W>
int launch_faln_t(const void* x, const void* r, const void* w, const void* b, void* y, void* so,
                  int64_t M, int64_t N, float eps, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  const T* xp = static_cast<const T*>(x);
  const T* rp = static_cast<const T*>(r);
  const W* wp = static_cast<const W*>(w);
  const W* bp = static_cast<const W*>(b);
  T* yp = static_cast<T*>(y);
  T* sp = static_cast<T*>(so);
  const bool rows_vec = (N % V == 0) && aligned16(x) && aligned16(r) && aligned16(y) &&
                        aligned16(so);
  const bool affine_vec = aligned16(w) && aligned16(b) && ((V * sizeof(W)) % 16 == 0);
  if (rows_vec) {
    int status = TILEOPS_OK;
    if (try_launch_ring<T, W>(xp, rp, wp, bp, yp, sp, M, N, eps, affine_vec, s, &status))
      return status;
    return launch_rows<T, W, V>(xp, rp, wp, bp, yp, sp, M, N, eps, affine_vec, s);
  }
  return launch_rows<T, W, 1>(xp, rp, wp, bp, yp, sp, M, N, eps, false, s);
}

}  // namespace
}  // namespace tileops

using namespace tileops;

extern "C" int tileops_fused_add_layer_norm_fwd(const void* x, const void* residual,
                                                const void* weight, const void* bias, void* y,
                                                void* residual_out, int64_t M, int64_t N,
                                                double eps, int dtype, int affine_dtype,
                                                void* stream) {
  if (M < 0 || N <= 0 || M > 0x7fffffffLL) return TILEOPS_EBADSHAPE;
  if (M == 0) return TILEOPS_OK;
  if (!x || !residual || !weight || !bias || !y || !residual_out) return TILEOPS_EINVAL;
  if (affine_dtype != dtype && affine_dtype != TILEOPS_DT_F32) return TILEOPS_EBADDTYPE;
  cudaStream_t s = as_stream(stream);
  const float e = static_cast<float>(eps);
  const bool f32_affine = affine_dtype == TILEOPS_DT_F32;
  switch (dtype) {
    case TILEOPS_DT_F32:
      return launch_faln_t<float, float>(x, residual, weight, bias, y, residual_out, M, N, e, s);
    case TILEOPS_DT_F16:
      return f32_affine ? launch_faln_t<__half, float>(x, residual, weight, bias, y,
                                                        residual_out, M, N, e, s)
                        : launch_faln_t<__half, __half>(x, residual, weight, bias, y,
                                                         residual_out, M, N, e, s);
    case TILEOPS_DT_BF16:
      return f32_affine ? launch_faln_t<__nv_bfloat16, float>(x, residual, weight, bias, y,
                                                               residual_out, M, N, e, s)
                        : launch_faln_t<__nv_bfloat16, __nv_bfloat16>(
                              x, residual, weight, bias, y, residual_out, M, N, e, s);
    default: return TILEOPS_EBADDTYPE;
  }
}
