// Shared helpers for the sm_100a TileOPs kernels: dtype traits, 16-byte
// vector access, launch geometry and argument checking for the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tileops_c.h"

namespace tileops {

// B200: 148 SMs.  Grids of streaming kernels are sized as a multiple of the
// SM count (queried once per device, with 148 as the default).
int sm_count();

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Map a launch error onto the ABI status.
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TILEOPS_OK : TILEOPS_ELAUNCH;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(int dt) {
  switch (dt) {
    case TILEOPS_DT_F32: return 4;
    case TILEOPS_DT_F16: return 2;
    case TILEOPS_DT_BF16: return 2;
    case TILEOPS_DT_BOOL: return 1;
    case TILEOPS_DT_U8: return 1;
    case TILEOPS_DT_I8: return 1;
    case TILEOPS_DT_I16: return 2;
    case TILEOPS_DT_I32: return 4;
    case TILEOPS_DT_I64: return 8;
    default: return 0;
  }
}

inline bool is_float_dtype(int dt) {
  return dt == TILEOPS_DT_F32 || dt == TILEOPS_DT_F16 || dt == TILEOPS_DT_BF16;
}

// ---- scalar conversion (fp32 opmath, round-to-nearest-even on store) ----
template <typename T>
struct Cvt;
template <>
struct Cvt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <>
struct Cvt<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <>
struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) {
    return __float2bfloat16_rn(v);
  }
};

// ---- packed fp32x2 arithmetic (sm_100a): one instruction, two lanes of work ----
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float ex2_approx_f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx_f(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- 16-byte vectors ----
// Streaming loads bypass L1 allocation (each byte is touched once); stores
// use the evict-first (.cs) hint so the output stream does not displace
// inputs still needed by other CTAs from L2.
// An empty volatile asm that claims to rewrite v: placed after a group of
// ld_stream calls, it keeps the compiler from hoisting any use of v (and so
// any arithmetic on it) above the last load of the group, so every load of
// the group is in flight before the first result is consumed.
__device__ __forceinline__ void after_loads(uint4& v) {
  asm volatile("" : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w));
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream8(void* p, uint2 v) {
  asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

// Elements of T in one 16-byte vector, and a union for lane access.
template <typename T>
union Pack16 {
  uint4 u;
  T e[16 / sizeof(T)];
};

// Grid for a grid-stride streaming loop: enough CTAs to cover `work` items
// of `per_cta` each, capped at `waves` full waves over the SMs.
// Division of 32-bit unsigned numerators by a divisor fixed at launch, as a
// multiply-high, an add and a shift (Granlund & Montgomery, "Division by
// invariant integers using multiplication", PLDI 1994): with
// s = ceil(log2 d) and m = floor(2^32 (2^s - d) / d) + 1,
// n / d = (umulhi(n, m) + n) >> s for every n < 2^32.
struct FastDivU32 {
  uint32_t d, m, s;
  explicit FastDivU32(uint32_t divisor = 1) : d(divisor), m(0), s(0) {
    while ((1ull << s) < d) ++s;
    m = static_cast<uint32_t>((((1ull << s) - d) << 32) / d + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return static_cast<uint32_t>(
        (static_cast<uint64_t>(__umulhi(n, m)) + n) >> s);
  }
};

// Grid of a single-pass streaming kernel: one CTA per `per_cta` units of
// work (at least one CTA, so block 0 can finish a ragged tail).
inline unsigned single_pass_grid(int64_t units, int64_t per_cta) {
  const int64_t g = (units + per_cta - 1) / per_cta;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

inline unsigned stream_grid(int64_t work, int64_t per_cta, int waves) {
  int64_t need = (work + per_cta - 1) / per_cta;
  int64_t cap = static_cast<int64_t>(sm_count()) * waves;
  if (need < 1) need = 1;
  return static_cast<unsigned>(need < cap ? need : cap);
}

}  // namespace tileops
