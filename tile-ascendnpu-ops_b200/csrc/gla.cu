// Gated linear attention (GLA), single-token decode step.
//
// Per (batch b, head h), state S (DK x DV), gate gk (DK), q, k (DK), v (DV):
//   S'[i, j] = exp(gk[i]) S[i, j] + k[i] v[j]          (fp32, stored in the dtype)
//   o[j]     = scale * sum_i q[i] S'[i, j]               (from the fp32 S')
// Reference: GLADecodeOp, examples/TileOPs/tileops/ops/linear_attention/gla_decode.py
// and its factory kernels/linear_attention/gla_decode/gla_decode_kernel/
// _gla_decode_kernel.py:57 (golden at :211-218).
//
// HBM-bound: the state is read once and written once (2 DK DV elements per
// (b, h)); everything else is O(DK + DV).  One CTA per (b, h) and slice of
// the DV columns (the columns of S are independent, so slicing needs no
// cross-CTA reduction; slices are added when B H alone would leave SMs idle).
// A thread owns one 16-byte packet column of its slice and walks rows
// i = r0, r0 + R, ...: it updates the packet in fp32, stores it rounded and
// accumulates q[i] S'[i, j] for its columns in registers; the row-group
// partials are then summed in a fixed order in shared memory.
#include <algorithm>

#include "common.cuh"

namespace tileops {
namespace {

constexpr int kGlaThreads = 256;

template <typename T>
struct GlaVec {
  static constexpr int kVec = 16 / sizeof(T);  // elements per 16-byte packet
};

// VEC = elements per access: GlaVec<T>::kVec (16-byte packets) or 1.  The
// slice has np <= 256 packets; threads are laid out as R = 256 / npad row
// groups of npad (np rounded up to a power of two) packet lanes, so every
// thread keeps one packet column and the column sums are deterministic.
template <typename T, int VEC>
__global__ void __launch_bounds__(kGlaThreads)
    gla_decode(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               const T* __restrict__ gk, const T* __restrict__ state, T* __restrict__ o,
               T* __restrict__ new_state, int DK, int DV, int pk_per_slice, int npad,
               float scale) {
  extern __shared__ float gsm[];
  float* qf = gsm;           // DK
  float* kf = qf + DK;       // DK
  float* ef = kf + DK;       // DK: exp(gk)
  float* vf = ef + DK;       // slice columns
  float* part = vf + pk_per_slice * VEC;  // [R][slice columns]
  const int bh = blockIdx.x;
  const int P = DV / VEC;                       // packets per row
  const int p0 = blockIdx.y * pk_per_slice;     // first packet of the slice
  const int np = min(pk_per_slice, P - p0);     // packets in the slice
  if (np <= 0) return;
  const int ncol = np * VEC;
  const int64_t vb = static_cast<int64_t>(bh) * DK;
  for (int i = threadIdx.x; i < DK; i += blockDim.x) {
    qf[i] = Cvt<T>::to_f(q[vb + i]);
    kf[i] = Cvt<T>::to_f(k[vb + i]);
    ef[i] = expf(Cvt<T>::to_f(gk[vb + i]));
  }
  for (int j = threadIdx.x; j < ncol; j += blockDim.x)
    vf[j] = Cvt<T>::to_f(v[static_cast<int64_t>(bh) * DV + p0 * VEC + j]);
  __syncthreads();

  const int R = kGlaThreads / npad;
  const int pc = threadIdx.x % npad, rg = threadIdx.x / npad;
  const int64_t sb = static_cast<int64_t>(bh) * DK * DV;
  if (pc < np) {
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.0f;
    float vr[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) vr[e] = vf[pc * VEC + e];
    // Rows rg, rg + R, ... in groups of kRowsInFlight: all loads of a group
    // are issued before any is used, so each thread keeps several 16-byte
    // reads in flight.
    constexpr int kRowsInFlight = 4;
    for (int row0 = rg; row0 < DK; row0 += R * kRowsInFlight) {
      T in[kRowsInFlight][VEC];
#pragma unroll
      for (int u = 0; u < kRowsInFlight; ++u) {
        const int row = row0 + u * R;
        if (row < DK) {
          const int64_t at = sb + static_cast<int64_t>(row) * DV + (p0 + pc) * VEC;
          if constexpr (VEC > 1) {
            *reinterpret_cast<uint4*>(in[u]) =
                __ldcs(reinterpret_cast<const uint4*>(state + at));
          } else {
            in[u][0] = state[at];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kRowsInFlight; ++u) {
        const int row = row0 + u * R;
        if (row >= DK) break;
        const int64_t at = sb + static_cast<int64_t>(row) * DV + (p0 + pc) * VEC;
        T out[VEC];
        const float e = ef[row], kr = kf[row], qr = qf[row];
#pragma unroll
        for (int x = 0; x < VEC; ++x) {
          const float sv = fmaf(e, Cvt<T>::to_f(in[u][x]), kr * vr[x]);
          out[x] = Cvt<T>::from_f(sv);
          acc[x] = fmaf(qr, sv, acc[x]);
        }
        if constexpr (VEC > 1) {
          __stcs(reinterpret_cast<uint4*>(new_state + at), *reinterpret_cast<const uint4*>(out));
        } else {
          new_state[at] = out[0];
        }
      }
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) part[rg * ncol + pc * VEC + e] = acc[e];
  }
  __syncthreads();
  for (int j = threadIdx.x; j < ncol; j += blockDim.x) {
    float sum = 0.0f;
    for (int g = 0; g < R; ++g) sum += part[g * ncol + j];
    o[static_cast<int64_t>(bh) * DV + p0 * VEC + j] = Cvt<T>::from_f(scale * sum);
  }
}

template <typename T>
int launch_gla(const void* q, const void* k, const void* v, const void* gk, const void* state,
               void* o, void* ns, int64_t BH, int DK, int DV, float scale, cudaStream_t s) {
  constexpr int kV = GlaVec<T>::kVec;
  const bool vec = DV % kV == 0 && aligned16(state) && aligned16(ns);
  const int vecw = vec ? kV : 1;
  const int P = DV / vecw;
  // Slices of the DV packets: enough CTAs for two per SM when B H is small,
  // at least 8 packets (128 bytes of a row) and at most 256 per slice.
  int nslice = (P + 255) / 256;
  const int64_t want = 2LL * sm_count();
  if (BH < want)
    nslice = std::max<int64_t>(nslice, std::min<int64_t>((want + BH - 1) / BH, (P + 7) / 8));
  const int per = (P + nslice - 1) / nslice;
  nslice = (P + per - 1) / per;
  int npad = 1;
  while (npad < per) npad <<= 1;
  const int R = kGlaThreads / npad;
  const size_t smem =
      (3 * static_cast<size_t>(DK) + static_cast<size_t>(per) * vecw * (1 + R)) * 4;
  if (smem > 200 * 1024) return TILEOPS_EBADSHAPE;
  const dim3 grid(static_cast<unsigned>(BH), static_cast<unsigned>(nslice));
  auto kv = vec ? gla_decode<T, kV> : gla_decode<T, 1>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kv, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return TILEOPS_ELAUNCH;
  kv<<<grid, kGlaThreads, smem, s>>>(static_cast<const T*>(q), static_cast<const T*>(k),
                                     static_cast<const T*>(v), static_cast<const T*>(gk),
                                     static_cast<const T*>(state), static_cast<T*>(o),
                                     static_cast<T*>(ns), DK, DV, per, npad, scale);
  return launch_status();
}

}  // namespace
}  // namespace tileops

using namespace tileops;

extern "C" int tileops_gla_decode_fwd(const void* q, const void* k, const void* v,
                                      const void* gk, const void* state, void* o,
                                      void* new_state, int64_t batch, int64_t heads,
                                      int64_t dim_k, int64_t dim_v, double scale, int dtype,
                                      void* stream) {
  if (batch < 0 || heads < 0 || dim_k <= 0 || dim_v <= 0 || dim_k > (1 << 16) ||
      dim_v > (1 << 16) || batch * heads > 0x7fffffffLL)
    return TILEOPS_EBADSHAPE;
  if (!is_float_dtype(dtype)) return TILEOPS_EBADDTYPE;
  const int64_t BH = batch * heads;
  if (BH == 0) return TILEOPS_OK;
  if (!q || !k || !v || !gk || !state || !o || !new_state) return TILEOPS_EINVAL;
  cudaStream_t s = as_stream(stream);
  const float sc = scale > 0.0 ? static_cast<float>(scale)
                               : static_cast<float>(1.0 / sqrt(static_cast<double>(dim_k)));
  const int DK = static_cast<int>(dim_k), DV = static_cast<int>(dim_v);
  switch (dtype) {
    case TILEOPS_DT_F32: return launch_gla<float>(q, k, v, gk, state, o, new_state, BH, DK, DV, sc, s);
    case TILEOPS_DT_F16: return launch_gla<__half>(q, k, v, gk, state, o, new_state, BH, DK, DV, sc, s);
    default: return launch_gla<__nv_bfloat16>(q, k, v, gk, state, o, new_state, BH, DK, DV, sc, s);
  }
}
