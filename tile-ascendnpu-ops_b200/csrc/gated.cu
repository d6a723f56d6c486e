// Gated activations: y[r, c] = act(x[r, c]) * x[r, N + c] for x of shape
// (M, 2N), y of shape (M, N).  act is the exact erf GELU or the tanh GELU.
//
// HBM-bound (3 * M * N * elem bytes per call).  The vector path gives each
// thread a 16-byte packet of the gate half and the matching packet of the
// value half (both coalesced across the warp, since packets of one warp are
// consecutive columns of one row), computes in fp32 and rounds once.  Four
// packet pairs are kept in flight per thread.  Rows whose width N is not a
// multiple of the packet, or misaligned pointers, take the scalar kernel.
//
// Reference: ops/elementwise/gelu_and_mul.py:42-125 and the test
// ref_program tests/ops/test_gelu_and_mul.py:63-76 (explicit erf, fp32);
// ops/elementwise/gelu_tanh_and_mul.py:43-126 with
// tests/ops/test_gelu_tanh_and_mul.py:64-86 (explicit tanh formula).
#include "common.cuh"

namespace tileops {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;  // packet pairs in flight per thread


// erf by Abramowitz & Stegun, Handbook of Mathematical Functions, formula
// 7.1.26 (Hastings' rational approximation): for a = |x|,
//   erf(a) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-a^2),
//   t = 1 / (1 + p a),  |error| <= 1.5e-7,
// and erf(-x) = -erf(x).  Branch-free: one reciprocal, one exp2, five FMAs,
// where a library erf spends ~30 instructions across two divergent ranges.
// Limits: erf(+-inf) = +-1 (t = 0, exp = 0) and NaN propagates.
__device__ __forceinline__ float erf_as7126(float x) {
  const float a = fabsf(x);
  const float t = rcp_approx_f(fmaf(0.3275911f, a, 1.0f));
  float poly = fmaf(t, 1.061405429f, -1.453152027f);
  poly = fmaf(t, poly, 1.421413741f);
  poly = fmaf(t, poly, -0.284496736f);
  poly = fmaf(t, poly, 0.254829592f);
  poly *= t;
  const float e = ex2_approx_f(-(a * a) * 1.4426950408889634f);  // exp(-a^2)
  return copysignf(fmaf(-poly, e, 1.0f), x);
}

// tanh(u) = 1 - 2 / (1 + exp(2u)); saturates to +-1 for large |u| and has an
// absolute error of a few 1e-7, which GELU multiplies by 0.5 g.
__device__ __forceinline__ float tanh_via_exp(float u) {
  return fmaf(-2.0f, rcp_approx_f(1.0f + ex2_approx_f(u * 2.8853900817779268f)), 1.0f);
}

struct GeluErfF {
  __device__ __forceinline__ float operator()(float g, float v) const {
    // 0.5 * g * (1 + erf(g * sqrt(0.5))) * v, same association as the reference.
    const float gelu = 0.5f * g * (1.0f + erf_as7126(g * 0.70710678118654752f));
    return gelu * v;
  }
};

struct GeluTanhF {
  __device__ __forceinline__ float operator()(float g, float v) const {
    // sqrt(2/pi) * (g + 0.044715 g^3), then 0.5 g (1 + tanh(inner)).
    const float inner = 0.79788456080286536f * (g + 0.044715f * (g * g * g));
    const float gelu = 0.5f * g * (1.0f + tanh_via_exp(inner));
    return gelu * v;
  }
};

// Packet p of the flattened (row, packet-in-row) index space sits in row
// p / pk_per_row; the division is a FastDivU32 when the index space fits in
// 32 bits (every shape up to 2^32 packets), a 64-bit division otherwise.
// Single pass: CTA b owns packets [b * kThreads * kUnroll, (b + 1) * ...),
// each thread kUnroll of them kThreads apart, all loads in flight together.
template <typename T, typename F, bool k32>
__global__ void __launch_bounds__(kThreads)
    gated_vec(const T* __restrict__ x, T* __restrict__ y, int64_t M, int64_t N, F f,
              FastDivU32 rowdiv) {
  constexpr int V = 16 / sizeof(T);
  const int64_t pk_per_row = N / V;
  const int64_t total = M * pk_per_row;
  auto row_of = [&](int64_t p) -> int64_t {
    if constexpr (k32) {
      return rowdiv.div(static_cast<uint32_t>(p));
    } else {
      return p / pk_per_row;
    }
  };
  const int64_t base = static_cast<int64_t>(blockIdx.x) * (kThreads * kUnroll) + threadIdx.x;
  Pack16<T> g[kUnroll], v[kUnroll];
  int64_t out_off[kUnroll];
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t p = base + u * kThreads;
    out_off[u] = -1;
    if (p < total) {
      const int64_t r = row_of(p);
      const int64_t c = (p - r * pk_per_row) * V;
      const T* row = x + r * 2 * N;
      g[u].u = ld_stream(row + c);
      v[u].u = ld_stream(row + N + c);
      out_off[u] = r * N + c;
    }
  }
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    after_loads(g[u].u);
    after_loads(v[u].u);
  }
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    if (out_off[u] >= 0) {
      Pack16<T> o;
#pragma unroll
      for (int e = 0; e < V; ++e)
        o.e[e] = Cvt<T>::from_f(f(Cvt<T>::to_f(g[u].e[e]), Cvt<T>::to_f(v[u].e[e])));
      st_stream(y + out_off[u], o.u);
    }
  }
}

template <typename T, typename F>
__global__ void __launch_bounds__(kThreads)
    gated_scalar(const T* __restrict__ x, T* __restrict__ y, int64_t M, int64_t N, F f) {
  const int64_t total = M * N;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += stride) {
    const int64_t r = i / N;
    const int64_t c = i - r * N;
    const T* row = x + r * 2 * N;
    y[i] = Cvt<T>::from_f(f(Cvt<T>::to_f(row[c]), Cvt<T>::to_f(row[N + c])));
  }
}

template <typename T, typename F>
int launch_gated_t(const void* x, void* y, int64_t M, int64_t N, F f, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  if (N % V == 0 && aligned16(x) && aligned16(y)) {
    const int64_t total = M * (N / V);
    const unsigned grid = single_pass_grid(total, kThreads * kUnroll);
    // 32-bit path: every packet index (< grid * kThreads * kUnroll) below 2^32.
    if (static_cast<int64_t>(grid) * kThreads * kUnroll <= (int64_t{1} << 32))
      gated_vec<T, F, true><<<grid, kThreads, 0, s>>>(
          xp, yp, M, N, f, FastDivU32(static_cast<uint32_t>(N / V)));
    else
      gated_vec<T, F, false><<<grid, kThreads, 0, s>>>(xp, yp, M, N, f, FastDivU32(1));
  } else {
    gated_scalar<T, F><<<stream_grid(M * N, kThreads, 8), kThreads, 0, s>>>(xp, yp, M, N, f);
  }
  return launch_status();
}

template <typename F>
int launch_gated(const void* x, void* y, int64_t M, int64_t N, int dtype, F f, void* stream) {
  if (M < 0 || N < 0) return TILEOPS_EBADSHAPE;
  if (M == 0 || N == 0) return TILEOPS_OK;
  if (!x || !y) return TILEOPS_EINVAL;
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case TILEOPS_DT_F32: return launch_gated_t<float>(x, y, M, N, f, s);
    case TILEOPS_DT_F16: return launch_gated_t<__half>(x, y, M, N, f, s);
    case TILEOPS_DT_BF16: return launch_gated_t<__nv_bfloat16>(x, y, M, N, f, s);
    default: return TILEOPS_EBADDTYPE;
  }
}

}  // namespace
}  // namespace tileops

using namespace tileops;

extern "C" int tileops_gelu_and_mul_fwd(const void* x, void* y, int64_t M, int64_t N, int dtype,
                                        void* stream) {
  return launch_gated(x, y, M, N, dtype, GeluErfF{}, stream);
}

extern "C" int tileops_gelu_tanh_and_mul_fwd(const void* x, void* y, int64_t M, int64_t N,
                                             int dtype, void* stream) {
  return launch_gated(x, y, M, N, dtype, GeluTanhF{}, stream);
}
