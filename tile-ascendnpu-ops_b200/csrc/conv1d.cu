// 1-D convolution over NCL tensors.
//
// Depthwise (groups == channels, one filter per channel) is the hot path:
//   out[n,c,o] = act(b[c] + sum_k w[c,k] * x[n,c,o*stride + k*dil - pad_left])
// with zero padding outside [0, l_in), fp32 accumulation and one rounding
// (reference: kernels/convolution/conv1d/conv1d_kernel/_conv1d_direct_kernel.py:10-40
// and its golden at :134-158).  The reference materialises a zero-padded
// copy of x in a host-allocated workspace (conv1d.py:570-578); here the
// padding is never stored, out-of-range taps read as zero in registers.
//
// Packet kernel (stride 1, dilation 1, small halo): each thread owns one
// 16-byte packet of the input row (8 bf16), the halo elements come from the
// neighbouring lanes' packets through warp shuffles, and only the two warp
// edge lanes fetch a neighbour packet from memory (an L2 hit).  x is read
// once and y written once in 16-byte packets: the kernel is HBM-bound at the
// algorithmic 2 * n*c*l * sizeof(T) bytes.  The causal Mamba form
// (k = 4, pad_left = 3) takes this path.
//
// Tiled kernel (any stride / dilation / k): the input window of a tile of
// outputs is staged in shared memory as fp32 and each thread produces
// outputs strided by the block size (bank-conflict free).
//
// Direct kernel (grouped / dense conv1d, the non-depthwise kernels of
// kernels/convolution/conv1d/conv1d.py:152-516): one output per thread,
// fp32 accumulation over c_in/groups * k taps.
#include "common.cuh"

namespace tileops {
namespace {

template <typename W>
__device__ __forceinline__ float ldw(const W* p) {
  return Cvt<W>::to_f(p[0]);
}

// SiLU(v) = v * sigmoid(v) = v / (1 + e^-v).  The fast exponential and
// division intrinsics (relative error ~2^-21) are far inside every tolerance
// this op is tested at (fp32 1e-4, 16-bit 1e-2); for v -> -inf the quotient
// correctly tends to -0.
__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == TILEOPS_ACT_SILU) return __fdividef(v, 1.0f + __expf(-v));
  return v;
}

// SiLU of two values with packed fp32x2 arithmetic: v * rcp(1 + 2^(-v log2 e))
// with ex2.approx / rcp.approx (relative error ~2^-21 each); large negative v
// gives 1 + e = inf, rcp = 0 and a signed zero.
__device__ __forceinline__ float2 silu2(float2 v) {
  const float2 m = fmul2(v, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  const float2 d = fadd2(make_float2(ex2_approx_f(m.x), ex2_approx_f(m.y)), make_float2(1.0f, 1.0f));
  return fmul2(v, make_float2(rcp_approx_f(d.x), rcp_approx_f(d.y)));
}

// ------------------------------------------------------------ packet path
constexpr int kPkThreads = 256;

// K taps and PAD left padding are compile-time so every window index is a
// constant and the 3-packet window lives in registers.  The window covers
// input positions [o0 - 8, o0 + 16), which holds every tap of the packet's
// 8 outputs when PAD <= 8 and K - PAD <= 9.
constexpr int kPkPerThread = 4;  // packets per thread (loads issued together)

template <typename T, typename W, int K, int PAD, int ACT>
__global__ void __launch_bounds__(kPkThreads)
    dwconv_packet(const T* __restrict__ x, const W* __restrict__ w, const W* __restrict__ bias,
                  T* __restrict__ y, int64_t C, int64_t l_in, int64_t l_out,
                  int64_t tiles_per_row) {
  constexpr int V = 8;  // elements per packet (16 bytes of a 2-byte type)
  static_assert(PAD <= V && K - PAD <= V + 1, "halo wider than one packet");
  const int64_t row = blockIdx.x / tiles_per_row;
  const int64_t tile = blockIdx.x - row * tiles_per_row;
  const int64_t c = row % C;
  const int lane = threadIdx.x & 31;
  const T* xr = x + row * l_in;
  T* yr = y + row * l_out;
  const int64_t in_pk = l_in / V;  // l_in % V == 0 on this path
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  // Packet i of this thread: consecutive lanes own consecutive packets, so
  // a lane's neighbours in the row are its neighbours in the warp.
  const int64_t pk0 = tile * (kPkThreads * kPkPerThread) + threadIdx.x;
  uint4 cur[kPkPerThread], edge[kPkPerThread];
#pragma unroll
  for (int i = 0; i < kPkPerThread; ++i) {
    const int64_t pk = pk0 + i * kPkThreads;
    cur[i] = (pk < in_pk) ? ld_stream(xr + pk * V) : zero;
  }
  // Warp-edge lanes fetch the packet beyond their warp's run (lane 0 the one
  // before, lane 31 the one after) together with the main loads; the
  // adjacent warp reads it at the same time, so it is an L2 hit.
#pragma unroll
  for (int i = 0; i < kPkPerThread; ++i) {
    const int64_t pk = pk0 + i * kPkThreads;
    edge[i] = zero;
    if (PAD > 0 && lane == 0 && pk >= 1 && pk - 1 < in_pk)
      edge[i] = __ldg(reinterpret_cast<const uint4*>(xr) + pk - 1);
    if (K - 1 - PAD > 0 && lane == 31 && pk + 1 < in_pk)
      edge[i] = __ldg(reinterpret_cast<const uint4*>(xr) + pk + 1);
  }
  float wk[K];
#pragma unroll
  for (int k = 0; k < K; ++k) wk[k] = ldw(w + c * K + k);
  const float bv = bias ? ldw(bias + c) : 0.0f;
#pragma unroll
  for (int i = 0; i < kPkPerThread; ++i) {
    const int64_t pk = pk0 + i * kPkThreads;
    uint4 prev, next;
    prev.x = __shfl_up_sync(0xffffffffu, cur[i].x, 1);
    prev.y = __shfl_up_sync(0xffffffffu, cur[i].y, 1);
    prev.z = __shfl_up_sync(0xffffffffu, cur[i].z, 1);
    prev.w = __shfl_up_sync(0xffffffffu, cur[i].w, 1);
    next.x = __shfl_down_sync(0xffffffffu, cur[i].x, 1);
    next.y = __shfl_down_sync(0xffffffffu, cur[i].y, 1);
    next.z = __shfl_down_sync(0xffffffffu, cur[i].z, 1);
    next.w = __shfl_down_sync(0xffffffffu, cur[i].w, 1);
    if (PAD > 0 && lane == 0) prev = edge[i];
    if (K - 1 - PAD > 0 && lane == 31) next = edge[i];
    const int64_t o0 = pk * V;
    if (o0 >= l_out) continue;
    float win[3 * V];  // win[t] = x[o0 - V + t]
    {
      Pack16<T> a, b2, d;
      a.u = prev;
      b2.u = cur[i];
      d.u = next;
#pragma unroll
      for (int t = 0; t < V; ++t) {
        win[t] = Cvt<T>::to_f(a.e[t]);
        win[V + t] = Cvt<T>::to_f(b2.e[t]);
        win[2 * V + t] = Cvt<T>::to_f(d.e[t]);
      }
    }
    // Outputs in pairs: the taps as packed fp32x2 FMAs.
    Pack16<T> out;
#pragma unroll
    for (int j = 0; j < V; j += 2) {
      float2 acc = make_float2(bv, bv);
#pragma unroll
      for (int k = 0; k < K; ++k)
        acc = ffma2(make_float2(wk[k], wk[k]),
                    make_float2(win[V + j + k - PAD], win[V + j + 1 + k - PAD]), acc);
      if constexpr (ACT == TILEOPS_ACT_SILU) acc = silu2(acc);
      out.e[j] = Cvt<T>::from_f(acc.x);
      out.e[j + 1] = Cvt<T>::from_f(acc.y);
    }
    if (o0 + V <= l_out) {
      st_stream(yr + o0, out.u);
    } else {
      for (int j = 0; j < V && o0 + j < l_out; ++j) yr[o0 + j] = out.e[j];
    }
  }
}

template <typename T, typename W, int K, int PAD>
int launch_packet(const T* x, const W* w, const W* b, T* y, int64_t c, int64_t l_in,
                  int64_t l_out, int act, int64_t rows, cudaStream_t s) {
  const int64_t pk_out = (l_out + 7) / 8;
  const int64_t per_cta = static_cast<int64_t>(kPkThreads) * kPkPerThread;
  const int64_t tiles = (pk_out + per_cta - 1) / per_cta;
  const int64_t grid = rows * tiles;
  if (grid > 0x7fffffffLL) return TILEOPS_EBADSHAPE;
  if (act == TILEOPS_ACT_SILU)
    dwconv_packet<T, W, K, PAD, TILEOPS_ACT_SILU><<<static_cast<unsigned>(grid), kPkThreads, 0, s>>>(
        x, w, b, y, c, l_in, l_out, tiles);
  else
    dwconv_packet<T, W, K, PAD, TILEOPS_ACT_NONE><<<static_cast<unsigned>(grid), kPkThreads, 0, s>>>(
        x, w, b, y, c, l_in, l_out, tiles);
  return launch_status();
}

// Returns 1 when (K, PAD) has a packet instantiation, after launching it.
template <typename T, typename W>
int try_packet(int K, int PAD, const T* x, const W* w, const W* b, T* y, int64_t c,
               int64_t l_in, int64_t l_out, int act, int64_t rows, cudaStream_t s,
               int* status) {
#define TILEOPS_PK(KK, PP)                                                                  \
  if (K == KK && PAD == PP) {                                                               \
    *status = launch_packet<T, W, KK, PP>(x, w, b, y, c, l_in, l_out, act, rows, s);        \
    return 1;                                                                               \
  }
  TILEOPS_PK(4, 3)  // causal Mamba conv (width 4)
  TILEOPS_PK(2, 1)
  TILEOPS_PK(3, 2)
  TILEOPS_PK(3, 1)
  TILEOPS_PK(3, 0)
  TILEOPS_PK(4, 0)
  TILEOPS_PK(5, 2)
  TILEOPS_PK(5, 4)
  TILEOPS_PK(7, 3)
  TILEOPS_PK(7, 6)
#undef TILEOPS_PK
  return 0;
}

// ------------------------------------------------------------- tiled path
constexpr int kTileThreads = 256;
constexpr int kTileOut = 1024;  // outputs per CTA

template <typename T, typename W>
__global__ void __launch_bounds__(kTileThreads)
    dwconv_tiled(const T* __restrict__ x, const W* __restrict__ w, const W* __restrict__ bias,
                 T* __restrict__ y, int64_t C, int64_t l_in, int64_t l_out, int K, int stride,
                 int dil, int pad_left, int act, int64_t tiles_per_row, int span) {
  extern __shared__ float sm[];  // [K weights][span inputs]
  float* ws = sm;
  float* xs = sm + K;
  const int64_t row = blockIdx.x / tiles_per_row;
  const int64_t tile = blockIdx.x - row * tiles_per_row;
  const int64_t c = row % C;
  const int64_t o0 = tile * kTileOut;
  const int64_t i0 = o0 * stride - pad_left;  // first input position of the tile's window
  const T* xr = x + row * l_in;
  for (int k = threadIdx.x; k < K; k += kTileThreads) ws[k] = ldw(w + c * K + k);
  for (int i = threadIdx.x; i < span; i += kTileThreads) {
    const int64_t p = i0 + i;
    xs[i] = (p >= 0 && p < l_in) ? Cvt<T>::to_f(xr[p]) : 0.0f;
  }
  __syncthreads();
  const float bv = bias ? ldw(bias + c) : 0.0f;
  T* yr = y + row * l_out;
  for (int j = threadIdx.x; j < kTileOut; j += kTileThreads) {
    const int64_t o = o0 + j;
    if (o >= l_out) break;
    float acc = bv;
    const int base = j * stride;
    for (int k = 0; k < K; ++k) acc = fmaf(ws[k], xs[base + k * dil], acc);
    yr[o] = Cvt<T>::from_f(apply_act(acc, act));
  }
}

// ------------------------------------------------------------ direct path
constexpr int kDirThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kDirThreads)
    conv1d_direct(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bias,
                  T* __restrict__ y, int64_t n, int64_t c_in, int64_t l_in, int64_t c_out,
                  int64_t l_out, int K, int stride, int pad_left, int dil, int64_t groups) {
  const int64_t total = n * c_out * l_out;
  const int64_t cig = c_in / groups, cog = c_out / groups;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * kDirThreads;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * kDirThreads + threadIdx.x; idx < total;
       idx += gstride) {
    const int64_t o = idx % l_out;
    const int64_t co = (idx / l_out) % c_out;
    const int64_t b = idx / (l_out * c_out);
    const int64_t g = co / cog;
    float acc = bias ? Cvt<T>::to_f(bias[co]) : 0.0f;
    const T* wr = w + co * cig * K;
    const T* xb = x + (b * c_in + g * cig) * l_in;
    for (int64_t ci = 0; ci < cig; ++ci) {
      const T* xr = xb + ci * l_in;
      for (int k = 0; k < K; ++k) {
        const int64_t p = o * stride + static_cast<int64_t>(k) * dil - pad_left;
        if (p >= 0 && p < l_in) acc = fmaf(Cvt<T>::to_f(wr[ci * K + k]), Cvt<T>::to_f(xr[p]), acc);
      }
    }
    y[idx] = Cvt<T>::from_f(acc);
  }
}

template <typename T, typename W>
int launch_dw_t(const void* x, const void* w, const void* bias, void* y, int64_t n, int64_t c,
                int64_t l_in, int64_t l_out, int K, int stride, int pad_left, int dil, int act,
                cudaStream_t s) {
  const T* xp = static_cast<const T*>(x);
  const W* wp = static_cast<const W*>(w);
  const W* bp = static_cast<const W*>(bias);
  T* yp = static_cast<T*>(y);
  const int64_t rows = n * c;
  const bool packet_ok = sizeof(T) == 2 && stride == 1 && dil == 1 && l_in % 8 == 0 &&
                         aligned16(x) && aligned16(y) && (l_out % 8 == 0);
  if (packet_ok) {
    int status = TILEOPS_OK;
    if (try_packet<T, W>(K, pad_left, xp, wp, bp, yp, c, l_in, l_out, act, rows, s, &status))
      return status;
  }
  const int64_t span64 = static_cast<int64_t>(kTileOut - 1) * stride +
                         static_cast<int64_t>(K - 1) * dil + 1;
  const int64_t smem = (span64 + K) * 4;
  if (smem <= 200 * 1024) {
    const int64_t tiles = (l_out + kTileOut - 1) / kTileOut;
    const int64_t grid = rows * tiles;
    if (grid > 0x7fffffffLL) return TILEOPS_EBADSHAPE;
    auto kern = dwconv_tiled<T, W>;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return TILEOPS_ELAUNCH;
    kern<<<static_cast<unsigned>(grid), kTileThreads, static_cast<size_t>(smem), s>>>(
        xp, wp, bp, yp, c, l_in, l_out, K, stride, dil, pad_left, act, tiles,
        static_cast<int>(span64));
    return launch_status();
  }
  return TILEOPS_EBADSHAPE;
}

}  // namespace
}  // namespace tileops

using namespace tileops;

extern "C" int tileops_conv1d_depthwise_fwd(const void* x, const void* w, const void* bias,
                                            void* y, int64_t n, int64_t c, int64_t l_in,
                                            int64_t l_out, int64_t k, int64_t stride,
                                            int64_t pad_left, int64_t dilation, int dtype,
                                            int w_dtype, int activation, void* stream) {
  if (n < 0 || c < 0 || l_in < 0 || l_out < 0 || k <= 0 || stride <= 0 || dilation <= 0 ||
      pad_left < 0 || k > 4096 || stride > 65536 || dilation > 65536 || pad_left > (1LL << 30))
    return TILEOPS_EBADSHAPE;
  if (activation != TILEOPS_ACT_NONE && activation != TILEOPS_ACT_SILU) return TILEOPS_EINVAL;
  if (n == 0 || c == 0 || l_out == 0) return TILEOPS_OK;
  if (!x || !w || !y) return TILEOPS_EINVAL;
  if (w_dtype != dtype && w_dtype != TILEOPS_DT_F32) return TILEOPS_EBADDTYPE;
  cudaStream_t s = as_stream(stream);
  const int K = static_cast<int>(k), st = static_cast<int>(stride), dl = static_cast<int>(dilation),
            pl = static_cast<int>(pad_left);
  const bool f32w = w_dtype == TILEOPS_DT_F32;
  switch (dtype) {
    case TILEOPS_DT_F16:
      return f32w ? launch_dw_t<__half, float>(x, w, bias, y, n, c, l_in, l_out, K, st, pl, dl,
                                               activation, s)
                  : launch_dw_t<__half, __half>(x, w, bias, y, n, c, l_in, l_out, K, st, pl, dl,
                                                activation, s);
    case TILEOPS_DT_BF16:
      return f32w ? launch_dw_t<__nv_bfloat16, float>(x, w, bias, y, n, c, l_in, l_out, K, st,
                                                      pl, dl, activation, s)
                  : launch_dw_t<__nv_bfloat16, __nv_bfloat16>(x, w, bias, y, n, c, l_in, l_out,
                                                              K, st, pl, dl, activation, s);
    case TILEOPS_DT_F32:
      return launch_dw_t<float, float>(x, w, bias, y, n, c, l_in, l_out, K, st, pl, dl,
                                       activation, s);
    default: return TILEOPS_EBADDTYPE;
  }
}

extern "C" int tileops_conv1d_direct_fwd(const void* x, const void* w, const void* bias, void* y,
                                         int64_t n, int64_t c_in, int64_t l_in, int64_t c_out,
                                         int64_t l_out, int64_t k, int64_t stride,
                                         int64_t pad_left, int64_t dilation, int64_t groups,
                                         int dtype, void* stream) {
  if (n < 0 || c_in <= 0 || l_in < 0 || c_out <= 0 || l_out < 0 || k <= 0 || stride <= 0 ||
      dilation <= 0 || pad_left < 0 || groups <= 0 || c_in % groups || c_out % groups ||
      k > (1 << 20) || stride > (1 << 20) || dilation > (1 << 20) || pad_left > (1LL << 30))
    return TILEOPS_EBADSHAPE;
  if (n == 0 || l_out == 0) return TILEOPS_OK;
  if (!x || !w || !y) return TILEOPS_EINVAL;
  cudaStream_t s = as_stream(stream);
  const int64_t total = n * c_out * l_out;
  const unsigned grid = stream_grid(total, kDirThreads, 16);
  const int K = static_cast<int>(k), st = static_cast<int>(stride), dl = static_cast<int>(dilation),
            pl = static_cast<int>(pad_left);
  switch (dtype) {
    case TILEOPS_DT_F16:
      conv1d_direct<__half><<<grid, kDirThreads, 0, s>>>(
          static_cast<const __half*>(x), static_cast<const __half*>(w),
          static_cast<const __half*>(bias), static_cast<__half*>(y), n, c_in, l_in, c_out, l_out,
          K, st, pl, dl, groups);
      break;
    case TILEOPS_DT_BF16:
      conv1d_direct<__nv_bfloat16><<<grid, kDirThreads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
          static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y), n, c_in, l_in,
          c_out, l_out, K, st, pl, dl, groups);
      break;
    case TILEOPS_DT_F32:
      conv1d_direct<float><<<grid, kDirThreads, 0, s>>>(
          static_cast<const float*>(x), static_cast<const float*>(w),
          static_cast<const float*>(bias), static_cast<float*>(y), n, c_in, l_in, c_out, l_out, K,
          st, pl, dl, groups);
      break;
    default: return TILEOPS_EBADDTYPE;
  }
  return launch_status();
}
