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
// Dense / grouped conv1d (the non-depthwise kernels of
// kernels/convolution/conv1d/conv1d.py:152-516), fp16 / bf16: an implicit
// GEMM on tcgen05 tensor cores.  Per (batch, group):
//   y[co, o] = b[co] + sum_r W[co, r] X[r, o],   r = ci * K + k,
//   X[r, o] = x[ci, o * stride + k * dil - pad_left]   (0 outside [0, l_in))
// M = output channels, N = output positions, K = c_in/groups * K.  One CTA
// (256 threads) per 128 x 128 output tile: the W rows of a 64-wide slice of r
// arrive by cp.async into a K-major swizzled tile, the matching im2col slice
// of x is gathered by the threads into an MN-major swizzled tile (consecutive
// threads read consecutive positions), two stages ring while one thread
// issues the MMAs; the fp32 accumulator lives in TMEM and the epilogue adds
// the bias and rounds once.  fp32 (and shapes beyond the grid limits) use the
// direct kernel: one output per thread, fp32 accumulation over the taps.
#include "common.cuh"
#include "sm100.cuh"

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

// ------------------------------------------------ implicit GEMM (tcgen05)
constexpr int kIgThreads = 256;
constexpr int kIgM = 128, kIgN = 128, kIgK = 64;  // tile of co x o, slice of r
constexpr int kIgStage = kIgM * kIgK * 2 + kIgK * kIgN * 2;  // A 16 KB + B 16 KB
constexpr int kIgSmem = 2 * kIgStage + 1024 /*bias*/ + 64 /*barriers*/ + 2 * kIgK * 16 /*row tables*/;

struct IgParams {
  const void* x;
  const void* x_end;  // one past the last element of x (bounds of the aligned loads)
  const void* w;
  const void* bias;
  void* y;
  int64_t c_in, l_in, c_out, l_out;
  int K, stride, pad_left, dil, groups;
  int cig, cog, R;  // channels per group, reduction length cig * K
  bool w_vec;       // W rows are 16-byte multiples and aligned: cp.async path
  bool x_win;       // stride 1 and x 16-byte aligned: windowed 16-byte gather
  bool y_pair;      // rows of y start 4-byte aligned: paired stores in the epilogue
  bool y_vec;       // rows of y start 16-byte aligned: 16-byte stores in the epilogue
  FastDivU32 div_k;
  int* err;
};

__device__ __forceinline__ uint32_t ig_swz(int r, int u) {
  return static_cast<uint32_t>(r * 128 + ((u ^ (r & 7)) << 4));
}

// Elements m..m+7 (16-bit) of the 16 elements in (a, b): the two 16-byte
// loads that cover an unaligned 8-element window, funnel-shifted into place.
__device__ __forceinline__ uint4 ig_window(const uint4& a, const uint4& b, int m) {
  auto fs = [](uint32_t lo, uint32_t hi) { return __funnelshift_r(lo, hi, 16); };
  switch (m) {
    case 0: return a;
    case 1: return make_uint4(fs(a.x, a.y), fs(a.y, a.z), fs(a.z, a.w), fs(a.w, b.x));
    case 2: return make_uint4(a.y, a.z, a.w, b.x);
    case 3: return make_uint4(fs(a.y, a.z), fs(a.z, a.w), fs(a.w, b.x), fs(b.x, b.y));
    case 4: return make_uint4(a.z, a.w, b.x, b.y);
    case 5: return make_uint4(fs(a.z, a.w), fs(a.w, b.x), fs(b.x, b.y), fs(b.y, b.z));
    case 6: return make_uint4(a.w, b.x, b.y, b.z);
    default: return make_uint4(fs(a.w, b.x), fs(b.x, b.y), fs(b.y, b.z), fs(b.z, b.w));
  }
}

// Three CTAs per SM: shared memory (two 32 KB stages each) allows three, and
// the register cap keeps the batched gather loads from halving that.
template <typename T>
__global__ void __launch_bounds__(kIgThreads, 3) conv1d_igemm(const IgParams p) {
  using namespace sm100;
  extern __shared__ uint8_t ig_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(ig_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* sbias = reinterpret_cast<float*>(sm + 2 * kIgStage);
  uint64_t* done = reinterpret_cast<uint64_t*>(sm + 2 * kIgStage + 1024);  // [2]
  uint64_t* all_done = done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(all_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Per stage: for the 64 reduction rows of the slice, the x offset of the
  // channel (ci * l_in) and the tap shift k * dil, or -1 past the end.
  int64_t* rtab = reinterpret_cast<int64_t*>(sm + 2 * kIgStage + 1024 + 64);  // [2][64][2]
  const uint32_t sb = smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int o0 = blockIdx.x * kIgN, co0 = blockIdx.y * kIgM;
  const int g = blockIdx.z % p.groups;
  const int64_t b = blockIdx.z / p.groups;
  const T* xg = static_cast<const T*>(p.x) + (b * p.c_in + static_cast<int64_t>(g) * p.cig) * p.l_in;
  const T* wg = static_cast<const T*>(p.w) + (static_cast<int64_t>(g) * p.cog + co0) * p.R;
  const int nchunk = (p.R + kIgK - 1) / kIgK;

  if (tid == 0) {
    mbar_init(&done[0], 1);
    mbar_init(&done[1], 1);
    mbar_init(all_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  if (tid < kIgM) {
    const int co = co0 + tid;
    sbias[tid] = (p.bias && co < p.cog)
                     ? Cvt<T>::to_f(static_cast<const T*>(p.bias)[static_cast<int64_t>(g) * p.cog + co])
                     : 0.0f;
  }

  // Slice c of r into stage c & 1: A = W[co0.., r0..] (K-major), B = X[r0.., o0..]
  // (MN-major, 64-position chunks 8 KB apart).
  auto stage = [&](int c) {
    uint8_t* st = sm + (c & 1) * kIgStage;
    const uint32_t sa = sb + (c & 1) * kIgStage;
    const int r0 = c * kIgK;
    if (p.w_vec) {
      for (int i = tid; i < kIgM * 8; i += kIgThreads) {
        const int row = i >> 3, u = i & 7;
        const int r = r0 + u * 8;
        const bool ok = co0 + row < p.cog && r < p.R;
        const T* src = ok ? wg + static_cast<int64_t>(row) * p.R + r : wg;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa + ig_swz(row, u)),
                     "l"(src), "r"(ok ? 16 : 0)
                     : "memory");
      }
    } else {
      // Element path: loads in batches of 16 in flight before their stores.
      constexpr int kPer = kIgM * kIgK / kIgThreads, kBatch = 16;
#pragma unroll 1
      for (int q0 = 0; q0 < kPer; q0 += kBatch) {
        T v[kBatch];
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
          const int i = tid + (q0 + q) * kIgThreads;
          const int row = i >> 6, r = r0 + (i & 63);
          v[q] = (co0 + row < p.cog && r < p.R) ? wg[static_cast<int64_t>(row) * p.R + r]
                                                : Cvt<T>::from_f(0.0f);
        }
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
          const int i = tid + (q0 + q) * kIgThreads;
          const int row = i >> 6, col = i & 63;
          *reinterpret_cast<T*>(st + ig_swz(row, col >> 3) + (col & 7) * 2) = v[q];
        }
      }
    }
    // B = X[r0.., o0..]: MN-major, 64-position chunks 8 KB apart.  (The row
    // table of this stage was written before the barrier preceding this call.)
    const int64_t* tb = rtab + (c & 1) * kIgK * 2;
    uint8_t* bt = st + kIgM * kIgK * 2;
    if (p.x_win) {
      // Row rr of the slice is the window x[ci, o0 - pad + k dil + (0..127)]:
      // thread -> 16-byte units i = tid + 256 q (row i / 16, positions
      // 8 (i % 16)..), each from two aligned 16-byte loads and a funnel shift;
      // units that cross a row edge or the end of x go element by element.
      // Every unit's aligned loads are issued before the first shared-memory
      // store (a store may not be reordered above a later generic load, so
      // loads interleaved with stores would cost one round trip per unit).
      constexpr int kUnits = kIgK * kIgN / 8 / kIgThreads;
      uint4 lo[kUnits], hi[kUnits];
      int mm[kUnits];
      bool fast[kUnits];
#pragma unroll
      for (int q = 0; q < kUnits; ++q) {
        const int i = tid + q * kIgThreads;
        const int rr = i >> 4, u = i & 15;
        const int64_t coff = tb[2 * rr];
        const int64_t pos = static_cast<int64_t>(o0) - p.pad_left + tb[2 * rr + 1] + u * 8;
        const uintptr_t src =
            reinterpret_cast<uintptr_t>(xg) + static_cast<uintptr_t>(coff + pos) * sizeof(T);
        const uintptr_t a16 = src & ~static_cast<uintptr_t>(15);
        mm[q] = static_cast<int>((src - a16) >> 1);
        fast[q] = coff >= 0 && pos >= 0 && pos + 8 <= p.l_in &&
                  a16 + 32 <= reinterpret_cast<uintptr_t>(p.x_end);
        lo[q] = hi[q] = make_uint4(0u, 0u, 0u, 0u);
        if (fast[q]) {
          lo[q] = *reinterpret_cast<const uint4*>(a16);
          if (mm[q]) hi[q] = *reinterpret_cast<const uint4*>(a16 + 16);
        }
      }
#pragma unroll
      for (int q = 0; q < kUnits; ++q) {
        const int i = tid + q * kIgThreads;
        const int rr = i >> 4, u = i & 15;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (fast[q]) {
          val = ig_window(lo[q], mm[q] ? hi[q] : lo[q], mm[q]);
        } else {
          const int64_t coff = tb[2 * rr];
          if (coff >= 0) {
            const int64_t pos = static_cast<int64_t>(o0) - p.pad_left + tb[2 * rr + 1] + u * 8;
            const T* src = xg + coff + pos;
            T* e = reinterpret_cast<T*>(&val);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              e[j] = (pos + j >= 0 && pos + j < p.l_in) ? src[j] : Cvt<T>::from_f(0.0f);
          }
        }
        // unit u of row rr: chunk u / 8 (8 KB apart), unit u % 8 of the 128-byte row
        *reinterpret_cast<uint4*>(bt + (u >> 3) * (kIgK * 128) + ig_swz(rr, u & 7)) = val;
      }
      return;
    }
    // Any stride: thread -> position o0 + (tid & 127), rows rr = tid >> 7, + 2, ...
    const int oo = tid & (kIgN - 1);
    const int64_t pos0 = static_cast<int64_t>(o0 + oo) * p.stride - p.pad_left;
    const bool o_ok = o0 + oo < p.l_out;
    uint8_t* bcol = bt + (oo >> 6) * (kIgK * 128) + (oo & 7) * 2;
    const int ucol = (oo & 63) >> 3;
    // This thread's kRows gather loads, in batches of 16 in flight before
    // their stores.
    constexpr int kRows = kIgK * kIgN / kIgThreads;
#pragma unroll 1
    for (int q0 = 0; q0 < kRows; q0 += 16) {
      T v[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const int rr = (tid >> 7) + (q0 + q) * (kIgThreads / kIgN);
        const int64_t coff = tb[2 * rr], shift = tb[2 * rr + 1];  // warp-uniform
        const int64_t pos = pos0 + shift;
        v[q] = (coff >= 0 && o_ok && pos >= 0 && pos < p.l_in) ? xg[coff + pos]
                                                               : Cvt<T>::from_f(0.0f);
      }
#pragma unroll
      for (int q = 0; q < 16; ++q)
        *reinterpret_cast<T*>(bcol + ig_swz((tid >> 7) + (q0 + q) * (kIgThreads / kIgN), ucol)) =
            v[q];
    }
  };

  auto write_table = [&](int c) {  // threads 0..63: row table of slice c
    if (tid < kIgK) {
      const int r = c * kIgK + tid;
      int64_t* t = rtab + (c & 1) * kIgK * 2 + 2 * tid;
      if (r < p.R) {
        const int ci = static_cast<int>(p.div_k.div(static_cast<uint32_t>(r)));
        t[0] = static_cast<int64_t>(ci) * p.l_in;
        t[1] = static_cast<int64_t>(r - ci * p.K) * p.dil;
      } else {
        t[0] = -1;
        t[1] = 0;
      }
    }
  };
  write_table(0);
  if (nchunk > 1) write_table(1);
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t idesc = idesc_f16_major(kIgM, kIgN, kBf16 ? 1 : 0, 0, 1);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  int issued = 0;
  for (int c = 0; c < nchunk; ++c) {
    const int buf = c & 1;
    if (c >= 2) {  // stage `buf` was read by slice c - 2's MMAs
      if (!mbar_wait(&done[buf], ((c - 2) >> 1) & 1, p.err, abort_flag)) ok = false;
      if (!__syncthreads_and(ok)) {
        ok = false;
        break;
      }
    }
    stage(c);
    asm volatile("cp.async.wait_all;" ::: "memory");
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Every thread is past stage(c): its table slot takes slice c + 2 (read
    // only after the barrier at the top of iteration c + 2).
    if (c + 2 < nchunk) write_table(c + 2);
    if (tid == 0) {
      const uint64_t a = smem_desc(sb + buf * kIgStage, 16, 1024);
      const uint64_t bd = smem_desc(sb + buf * kIgStage + kIgM * kIgK * 2, kIgK * 128, 1024);
#pragma unroll
      for (int kk = 0; kk < kIgK / 16; ++kk)
        mma_f16_ss(tmem, desc_advance(a, kk * 32), desc_advance(bd, kk * 16 * 128), idesc,
                   (c > 0 || kk > 0) ? 1u : 0u);
      mma_commit(&done[buf]);
    }
    issued = c + 1;
  }
  if (tid == 0) mma_commit(all_done);
  const bool fin = mbar_wait(all_done, 0, p.err, abort_flag, !ok);
  tc_fence_after();
  // Uniform across the CTA: the epilogue below synchronises.
  if (__syncthreads_and(ok && fin && issued == nchunk)) {
    // TMEM lane = output channel co0 + 32 (w % 4) + lane; warps w and w + 4
    // take positions [0, 64) and [64, 128).  The rounded tile is staged in
    // the freed stage buffers as [128 co][128 o] (16-byte units swizzled by
    // row) and written row by row by consecutive threads, coalesced whatever
    // the alignment of the rows in y.
    const int row = (warp & 3) * 32 + (tid & 31);
    const int cb = (warp >> 2) * 64;
    const uint32_t lane = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float bv = sbias[row];
    uint8_t* stg = sm;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t v[32];
      tmem_ld32(tmem + lane + cb + h * 32, v);
      tmem_wait_ld_regs(v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 pk;
        uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const T lo = Cvt<T>::from_f(__uint_as_float(v[8 * q + 2 * e]) + bv);
          const T hi = Cvt<T>::from_f(__uint_as_float(v[8 * q + 2 * e + 1]) + bv);
          pw[e] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&lo)) |
                  (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
        }
        const int u = (cb + h * 32) / 8 + q;  // 16-byte unit of the row (16 per row)
        *reinterpret_cast<uint4*>(stg + row * 256 + ((u ^ (row & 15)) << 4)) = pk;
      }
    }
    __syncthreads();
    const int nrow = min(kIgM, p.cog - co0), ncol = min(kIgN, static_cast<int>(p.l_out - o0));
    T* ybase = static_cast<T*>(p.y) +
               (b * p.c_out + static_cast<int64_t>(g) * p.cog + co0) * p.l_out + o0;
    // Element pairs as 4-byte stores when every row starts 4-byte aligned
    // (y aligned, l_out and o0 even): lane l writes columns 2l, 2l + 1,
    // 2l + 64, 2l + 65 of its warp's rows; otherwise single elements.
    const bool pairs = p.y_pair && (ncol & 1) == 0;
    if (p.y_vec) {
      // 16-byte units: half-warp per row, two rows per warp instruction
      // (ncol is a multiple of 8 here since l_out and o0 are).
      const int u = tid & 15;
      for (int rr = 2 * warp + ((tid >> 4) & 1); rr < nrow; rr += kIgThreads / 16) {
        if (u * 8 < ncol)
          *reinterpret_cast<uint4*>(ybase + static_cast<int64_t>(rr) * p.l_out + u * 8) =
              *reinterpret_cast<const uint4*>(stg + rr * 256 + ((u ^ (rr & 15)) << 4));
      }
    } else {
      for (int rr = warp; rr < nrow; rr += kIgThreads / 32) {
        T* yr = ybase + static_cast<int64_t>(rr) * p.l_out;
        const uint8_t* sr = stg + rr * 256;
        if (pairs) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = 2 * (tid & 31) + 64 * h;
            if (c < ncol) {
              const uint32_t v =
                  *reinterpret_cast<const uint32_t*>(sr + (((c >> 3) ^ (rr & 15)) << 4) + (c & 7) * 2);
              *reinterpret_cast<uint32_t*>(yr + c) = v;
            }
          }
        } else {
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const int c = (tid & 31) + 32 * h;
            if (c < ncol)
              yr[c] = *reinterpret_cast<const T*>(sr + (((c >> 3) ^ (rr & 15)) << 4) + (c & 7) * 2);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

template <typename T>
int launch_igemm(const void* x, const void* w, const void* bias, void* y, int64_t n,
                 int64_t c_in, int64_t l_in, int64_t c_out, int64_t l_out, int K, int stride,
                 int pad_left, int dil, int64_t groups, cudaStream_t s) {
  IgParams p;
  p.x = x;
  p.x_end = static_cast<const T*>(x) + n * c_in * l_in;
  p.w = w;
  p.bias = bias;
  p.y = y;
  p.c_in = c_in;
  p.l_in = l_in;
  p.c_out = c_out;
  p.l_out = l_out;
  p.K = K;
  p.stride = stride;
  p.pad_left = pad_left;
  p.dil = dil;
  p.groups = static_cast<int>(groups);
  p.cig = static_cast<int>(c_in / groups);
  p.cog = static_cast<int>(c_out / groups);
  p.R = p.cig * K;
  p.w_vec = p.R % 8 == 0 && aligned16(w);
  p.x_win = stride == 1 && aligned16(x);
  p.y_pair = (reinterpret_cast<uintptr_t>(y) & 3u) == 0 && l_out % 2 == 0;
  p.y_vec = aligned16(y) && l_out % 8 == 0;
  p.div_k = FastDivU32(static_cast<uint32_t>(K));
  p.err = device_error_ptr();
  auto k = conv1d_igemm<T>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kIgSmem + 1024) !=
      cudaSuccess)
    return TILEOPS_ELAUNCH;
  const dim3 grid(static_cast<unsigned>((l_out + kIgN - 1) / kIgN),
                  static_cast<unsigned>((p.cog + kIgM - 1) / kIgM),
                  static_cast<unsigned>(n * groups));
  k<<<grid, kIgThreads, kIgSmem + 1024, s>>>(p);
  return launch_status();
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
  // 16-bit: the tcgen05 implicit GEMM when the grid and the 32-bit index
  // arithmetic of its gather fit.
  const int64_t cig = c_in / groups;
  if ((dtype == TILEOPS_DT_F16 || dtype == TILEOPS_DT_BF16) && n * groups <= 65535 &&
      (c_out / groups + kIgM - 1) / kIgM <= 65535 && (l_out + kIgN - 1) / kIgN <= 0x7fffffffLL &&
      cig * k <= 0x7fffffffLL && l_out * stride <= (1LL << 40)) {
    const int K = static_cast<int>(k), st = static_cast<int>(stride),
              dl = static_cast<int>(dilation), pl = static_cast<int>(pad_left);
    return dtype == TILEOPS_DT_BF16
               ? launch_igemm<__nv_bfloat16>(x, w, bias, y, n, c_in, l_in, c_out, l_out, K, st,
                                             pl, dl, groups, s)
               : launch_igemm<__half>(x, w, bias, y, n, c_in, l_in, c_out, l_out, K, st, pl, dl,
                                      groups, s);
  }
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
