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
// One CTA (256 threads; three per SM on the tensor-copy path, two on the
// cp.async path) per (b, c, h, 128-row tile of the chunk); row l0 + r of the
// tile is TMEM lane r.  Both terms are tcgen05 MMAs (M = 128,
// N = P, kind::f16, fp32 accumulators in TMEM):
//   D1 = C_tile [128 x N] . prev^T        A K-major (C rows), B K-major (prev
//                                          rows p, converted fp32 -> dtype)
//   D2 = W [128 x s] . x [s x P]          A = W built per 64-key block in
//                                          shared memory, B MN-major (x rows s)
// with W[l, s] = cb[l, s] exp(dA[l] - dA[s]) dt[s] for s <= l (< Q), else 0.
// The cb rows of a key block land in shared memory and are turned into W in
// place.  For bf16 on the tensor-copy path, when the tile's decay range
// allows it, the decay is split instead: the x rows are scaled by
// exp(ref - dA[s]) dt[s], cb enters the MMA as loaded (masked only in the
// blocks that reach the diagonal) and row l of D2 is multiplied by
// exp(dA[l] - ref) in the epilogue.  cb / W and x blocks are triple-buffered
// and requested two blocks ahead; buffers the history operands occupy are
// reused once the history MMA has read them (SsdLayout).  Loads: with chunk
// length, d_head and d_state multiples of 64 the C tile, x and cb blocks are
// tensor copies (one thread, mbarrier completion), otherwise 16-byte cp.async
// from every thread (zero fill past the chunk / past N).  Epilogue:
// out = exp(dA[l]) D1 + r_l D2 from TMEM (r_l the row factor, 1 for the W
// build), staged in shared memory and written by tensor stores (chunk length a
// multiple of 128) or by row-wise vector stores.
// Every mbarrier wait (sm100::mbar_wait) checks a 2 s limit between its
// try_wait polls; a phase that completes late sets the device error flag, the
// MMAs issued so far are drained and TMEM is freed before returning.
#include <cudaTypedefs.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace tileops {
namespace {

using namespace sm100;

constexpr int kSsdThreads = 256;
constexpr int kSsdRowGroups = kSsdThreads / 8;  // rows of a W block handled together
constexpr int kSsdRows = 128;   // chunk rows per CTA (MMA M)
constexpr int kSsdKBlk = 64;    // keys per W / x block
constexpr int kSsdMaxN = 256;   // d_state
constexpr int kSsdMaxP = 128;   // d_head
constexpr int kSsdMaxQ = 1024;  // chunk length

// 16-byte unit u of 128-byte row r of a swizzled 64-column tile.
__device__ __forceinline__ uint32_t ssd_swz(int r, int u) {
  return static_cast<uint32_t>(r * 128 + ((u ^ (r & 7)) << 4));
}

constexpr int kSsdBarBytes = 128;  // the SsdBars block at the end of the layout

// Shared-memory layout, sized per call (offsets in bytes from a 1 KB-aligned
// base, every tile 1 KB aligned): C [128][nc64] and prev [P][nc64] K-major
// (nc64 = d_state rounded up to 64-column chunks) for the history MMA, three
// key-block buffers, each a cb / W block [128][64] and an x block [64][pc64]
// MN-major (pc64 = d_head rounded up to 64), dA (fp32) and dt (the 16-bit
// type) of the chunk, the per-block dA ranges, the barriers.
//   ring = false (cp.async path): two dedicated cb / W blocks, three dedicated
//     x blocks; the third cb / W block lives in the C tile once the history
//     MMA has read it.
//   ring = true (tensor-copy path): buffer 0 is dedicated; buffers 1 and 2
//     (a cb block and its x block each) reuse the C / prev region once the
//     history MMA has read it, which keeps the bf16 / fp16 d_head 64,
//     d_state 128, chunk 256 case at 76.6 KB, three CTAs per SM.
struct SsdLayout {
  int c, prev, w, x, da, dt, rng, bar, bytes;
  int x_stride;  // ring = false: bytes of one x block
  int slot;      // ring = true: bytes of one buffer (cb block + x block)
  int ring0;     // ring = true: offset of buffer 0
  bool ring;
  __host__ __device__ static int up1k(int v) { return (v + 1023) & ~1023; }
  __host__ __device__ SsdLayout(int P, int N, int Q, bool ring_) : ring(ring_) {
    const int nc64 = ((N + 63) / 64) * 64, pc64 = ((P + 63) / 64) * 64;
    constexpr int kCb = kSsdRows * kSsdKBlk * 2;
    c = 0;
    prev = up1k(c + kSsdRows * nc64 * 2);
    const int hist_end = up1k(prev + P * nc64 * 2);
    x_stride = kSsdKBlk * pc64 * 2;
    slot = kCb + x_stride;
    int end;
    if (ring) {
      ring0 = hist_end > 2 * slot ? hist_end : 2 * slot;  // buffers 1, 2 below it
      w = x = -1;
      end = ring0 + slot;
    } else {
      ring0 = -1;
      w = hist_end;
      x = w + 2 * kCb;
      end = x + 3 * x_stride;
    }
    // dA (fp32) and dt (16-bit) of the chunk, each starting on a 16-byte
    // boundary (the W build reads 8 keys of each at once).
    da = end;
    dt = da + ((Q * 4 + 15) & ~15);
    // per 64-key block: min, max of dA, and 1.0f if its dA and dt are all finite (3 x 16 floats)
    rng = dt + ((Q * 2 + 15) & ~15);
    bar = rng + 3 * 16 * 4;
    bytes = bar + kSsdBarBytes;
  }
  // cb / W block of buffer i.  ring = false: 0, 1 dedicated, 2 the C tile.
  __host__ __device__ int cbuf(int i) const {
    if (ring) return i == 0 ? ring0 : (i - 1) * slot;
    return i == 2 ? c : w + i * (kSsdRows * kSsdKBlk * 2);
  }
  // x block of buffer i.
  __host__ __device__ int xbuf(int i) const {
    return ring ? cbuf(i) + kSsdRows * kSsdKBlk * 2 : x + i * x_stride;
  }
  // Output staging after the last MMA: a region of at least 128 x P fp32.
  __host__ __device__ int stage() const { return ring ? 0 : w; }
};

struct SsdBars {
  uint64_t full[3];      // tensor-copy path: x and cb of the block in buffer i landed
  uint64_t c_full;       // tensor-copy path: the C tile landed
  uint64_t blk_done[3];  // MMAs of the cb / W and x blocks in buffer i completed
  uint64_t d1_done;      // the history MMA completed (the C tile may be reused)
  uint64_t all_done;     // every MMA completed
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(SsdBars) <= kSsdBarBytes, "SsdBars outgrew its layout slot");

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
// Every committed group but the most recent one has completed.
__device__ __forceinline__ void cp_async_wait_prev() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
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
  FastDivU32 div_c;  // npad / 8: 16-byte units of a C / prev row
  FastDivU32 div_x;  // P / 8: 16-byte units of an x row
  FastDivU32 div_o;  // P / 4: 16-byte units of an fp32 output row
  int* err;
};

// kTma: the C tile, x blocks and cb blocks are brought by tensor copies
// (one thread, completion on mbarriers) instead of 16-byte cp.async from
// every thread, which keeps the SM's load / shared-memory pipeline free for
// the W build; requires chunk length, d_head and d_state multiples of 64.
// With kTma and a chunk length that is a multiple of 128 (no row tile
// reaches into the next chunk) the output leaves by tensor stores too.
template <typename T, bool kTma>
__global__ void __launch_bounds__(kSsdThreads, kTma ? 3 : 2)
    ssd_chunk_scan(const SsdParams p, const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_c,
                   const __grid_constant__ CUtensorMap tm_cb,
                   const __grid_constant__ CUtensorMap tm_out) {
  const SsdLayout L(p.P, p.N, p.Q, kTma);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  SsdBars* bars = reinterpret_cast<SsdBars*>(sm + L.bar);
  volatile int* abort_flag = &bars->abort_flag;
  float* sdA = reinterpret_cast<float*>(sm + L.da);
  T* sdt = reinterpret_cast<T*>(sm + L.dt);
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
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->blk_done[i], 1);
    }
    mbar_init(&bars->c_full, 1);
    mbar_init(&bars->d1_done, 1);
    mbar_init(&bars->all_done, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  // TMEM: D1 at column 0, D2 at column P rounded up to 64.
  const uint32_t tmem_cols = ((P + 63) & ~63) * 2 <= 128 ? 128u : 256u;
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, tmem_cols);
    tmem_relinquish();
  }

  const int64_t hc = (static_cast<int64_t>(b) * p.H + h) * p.NC + c;
  const T* xg = static_cast<const T*>(p.x);
  const T* cbg = static_cast<const T*>(p.cb) +
                 ((static_cast<int64_t>(b) * p.NC + c) * p.G + g) * static_cast<int64_t>(Q) * Q;
  const float* pg = p.prev + ((static_cast<int64_t>(b) * p.NC + c) * p.H + h) * P * N;
  const int pupr = npad / 8, ptotal = P * pupr;  // 16-byte units of prev rows (as dtype)

  // ---- prologue: every global load of the CTA's first two blocks in flight
  // at once (prev and dA / dt into registers, C, x and cb by cp.async).
  // prev packets per thread and round: four at three CTAs per SM (80 registers)
  constexpr int kPrevPer = kTma ? 4 : 8;
  float4 va[kPrevPer], vb[kPrevPer];  // this thread's prev packets of a round (fp32)
  auto load_prev = [&](int base) {
#pragma unroll
    for (int k = 0; k < kPrevPer; ++k) {
      const int i = base + k * kSsdThreads + tid;
      va[k] = vb[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (i < ptotal) {
        const int r = static_cast<int>(p.div_c.div(i)), n = (i - r * pupr) * 8;
        if (n < N) {
          const float* src = pg + static_cast<int64_t>(r) * N + n;
          va[k] = __ldcs(reinterpret_cast<const float4*>(src));
          vb[k] = __ldcs(reinterpret_cast<const float4*>(src + 4));
        }
      }
    }
  };
  auto store_prev = [&](int base) {  // -> dtype, K-major [p][n]
#pragma unroll
    for (int k = 0; k < kPrevPer; ++k) {
      const int i = base + k * kSsdThreads + tid;
      if (i < ptotal) {
        const int r = static_cast<int>(p.div_c.div(i)), n = (i - r * pupr) * 8;
        uint4 pk;
        pk.x = pack16<T>(va[k].x, va[k].y);
        pk.y = pack16<T>(va[k].z, va[k].w);
        pk.z = pack16<T>(vb[k].x, vb[k].y);
        pk.w = pack16<T>(vb[k].z, vb[k].w);
        *reinterpret_cast<uint4*>(sm + L.prev + (n >> 6) * (P * 128) +
                                  ssd_swz(r, (n & 63) >> 3)) = pk;
      }
    }
  };
  load_prev(0);
  constexpr int kMaxQPerThread = kSsdMaxQ / kSsdThreads;
  float rdA[kMaxQPerThread];
  T rdt[kMaxQPerThread];
#pragma unroll
  for (int k = 0; k < kMaxQPerThread; ++k) {
    const int i = tid + k * kSsdThreads;
    if (i < Q) {
      rdA[k] = p.dA[hc * Q + i];
      rdt[k] = static_cast<const T*>(p.dt)[hc * Q + i];
    }
  }

  // Thread layout of a cb / W block: packet column cpk (keys 8 cpk.. of the
  // block) of rows rg + kSsdRowGroups it; the thread that copies a packet is
  // the one that turns it into W, so no barrier separates the two.
  const int cpk = tid & 7, rg = tid >> 3;
  const bool cbvec = (Q & 7) == 0;
  auto issue_cb = [&](int j) {  // cb rows of key block j -> cb / W buffer j % 3
    const int sc = j * kSsdKBlk + cpk * 8;
    uint8_t* dst = sm + L.cbuf(j % 3);
#pragma unroll
    for (int it = 0; it < kSsdRows / kSsdRowGroups; ++it) {
      const int r = rg + kSsdRowGroups * it;
      const int l = l0 + r;
      // Packets wholly above the diagonal, past the chunk, or of rows past
      // the chunk are zero.
      const bool ok = l < Q && sc <= l && sc < Q;
      const T* row = cbg + static_cast<int64_t>(ok ? l : 0) * Q + (ok ? sc : 0);
      if (cbvec) {
        cp_async16(sb + L.cbuf(j % 3) + ssd_swz(r, cpk), row, ok);
      } else {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (ok) {
          T* cv = reinterpret_cast<T*>(&v);
#pragma unroll
          for (int e = 0; e < 8; ++e) cv[e] = sc + e < Q ? row[e] : Cvt<T>::from_f(0.0f);
        }
        *reinterpret_cast<uint4*>(dst + ssd_swz(r, cpk)) = v;
      }
    }
  };
  auto issue_x = [&](int j) {  // x rows of key block j -> buffer j % 3 (cp.async)
    const int s0 = j * kSsdKBlk, upr = P / 8;
    for (int i = tid; i < kSsdKBlk * upr; i += kSsdThreads) {
      const int r = static_cast<int>(p.div_x.div(i)), u = i - r * upr;
      const int s = s0 + r, pc = u * 8;
      const bool ok = s < Q;
      const T* src = xg + ((static_cast<int64_t>(b) * S + c * Q + (ok ? s : 0)) * p.H + h) * P + pc;
      cp_async16(sb + L.xbuf(j % 3) + (pc >> 6) * (kSsdKBlk * 128) +
                     ssd_swz(r, (pc & 63) >> 3),
                 src, ok);
    }
  };
  // Tensor-copy path: block j's x rows and cb rows -> buffers j % 3 (thread 0).
  const int bcg = (b * p.NC + c) * p.G + g;
  int armed[3] = {-1, -1, -1};  // thread 0: last block whose copies each buffer awaits
  auto tma_blk = [&](int j) {
    const int i = j % 3;
    mbar_arrive_expect_tx(&bars->full[i],
                          static_cast<uint32_t>(P * kSsdKBlk * 2 + kSsdRows * kSsdKBlk * 2));
    for (int pc = 0; pc < P; pc += 64)
      tma_load_4d(sm + L.xbuf(i) + (pc >> 6) * (kSsdKBlk * 128), &tm_x,
                  &bars->full[i], pc, h, c * Q + j * kSsdKBlk, b);
    tma_load_3d(sm + L.cbuf(i), &tm_cb, &bars->full[i], j * kSsdKBlk, l0, bcg);
    armed[i] = j;
  };
  if constexpr (kTma) {
    if (tid == 0) {
      prefetch_tensormap(&tm_x);
      prefetch_tensormap(&tm_c);
      prefetch_tensormap(&tm_cb);
      mbar_arrive_expect_tx(&bars->c_full, static_cast<uint32_t>(kSsdRows * N * 2));
      for (int n0 = 0; n0 < N; n0 += 64)
        tma_load_4d(sm + L.c + (n0 >> 6) * (kSsdRows * 128), &tm_c, &bars->c_full, n0, g,
                    c * Q + l0, b);
      tma_blk(0);  // buffers 1 and 2 hold C / prev until the history MMA has read them
    }
  } else {
    const T* Cg = static_cast<const T*>(p.C);
    const int upr = npad / 8;  // 16-byte units per row
    for (int i = tid; i < kSsdRows * upr; i += kSsdThreads) {
      const int r = static_cast<int>(p.div_c.div(i)), u = i - r * upr;
      const int l = l0 + r, n = u * 8;
      const bool ok = l < Q && n < N;
      const T* src = Cg + ((static_cast<int64_t>(b) * S + c * Q + (ok ? l : 0)) * p.G + g) * N +
                     (ok ? n : 0);
      cp_async16(sb + L.c + (n >> 6) * (kSsdRows * 128) + ssd_swz(r, (n & 63) >> 3), src, ok);
    }
    issue_x(0);
    issue_cb(0);
    cp_async_commit();  // group 0: the C tile, x and cb of block 0
    if (nblk > 1) {
      issue_x(1);
      issue_cb(1);
      cp_async_commit();  // group 1: x and cb of block 1
    }
  }
  // dA is kept in log2 units: exp(a - b) = ex2(a' - b').
#pragma unroll
  for (int k = 0; k < kMaxQPerThread; ++k) {
    const int i = tid + k * kSsdThreads;
    if (i < Q) {
      sdA[i] = rdA[k] * 1.4426950408889634f;
      sdt[i] = rdt[k];
    }
  }
  store_prev(0);
  for (int base = kPrevPer * kSsdThreads; base < ptotal; base += kPrevPer * kSsdThreads) {
    load_prev(base);  // shapes with more than 8 prev packets per thread
    store_prev(base);
  }
  if constexpr (!kTma) {
    if (nblk > 1) cp_async_wait_prev();  // group 0 landed (this thread's copies)
    else cp_async_wait_all();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();  // C, prev, sdA / sdt, block 0 visible; barriers initialised
  tc_fence_after();

  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t id_kk = idesc_f16_major(kSsdRows, P, kBf16 ? 1 : 0, 0, 0);
  const uint32_t id_kmn = idesc_f16_major(kSsdRows, P, kBf16 ? 1 : 0, 0, 1);
  const uint32_t tmem = bars->tmem_base;
  const uint32_t p64 = static_cast<uint32_t>((P + 63) & ~63);
  const uint32_t t_d1 = tmem, t_d2 = tmem + p64;
  bool ok = true;
  if (tid == 0) {  // history: D1 = C prev^T
    if constexpr (kTma) ok = mbar_wait(&bars->c_full, 0, p.err, abort_flag);
    const uint64_t a = smem_desc(sb + L.c, 16, 1024);
    const uint64_t bd = smem_desc(sb + L.prev, 16, 1024);
    if (ok) {
      tc_fence_after();
      for (int kk = 0; kk < npad / 16; ++kk)
        mma_f16_ss(t_d1, desc_advance(a, (kk >> 2) * (kSsdRows * 128) + (kk & 3) * 32),
                   desc_advance(bd, (kk >> 2) * (P * 128) + (kk & 3) * 32), id_kk, kk > 0);
    }
    mma_commit(&bars->d1_done);
  }
  {
    // min / max of dA over each 64-key block (warp w: blocks w, w + 8, ...),
    // and whether every dA and dt of the block is finite
    float* rng = reinterpret_cast<float*>(sm + L.rng);
    const int lane = tid & 31;
    for (int jb = warp; jb * kSsdKBlk < Q; jb += kSsdThreads / 32) {
      float mn = INFINITY, mx = -INFINITY;
      bool fin = true;
      for (int k = lane; k < kSsdKBlk; k += 32) {
        const int s = jb * kSsdKBlk + k;
        if (s < Q) {
          mn = fminf(mn, sdA[s]);
          mx = fmaxf(mx, sdA[s]);
          fin = fin && fabsf(sdA[s]) < INFINITY && fabsf(Cvt<T>::to_f(sdt[s])) < INFINITY;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      }
      fin = __all_sync(0xffffffffu, fin);
      if (lane == 0) {
        rng[jb] = mn;
        rng[16 + jb] = mx;
        rng[32 + jb] = fin ? 1.0f : 0.0f;
      }
    }
  }
  __syncthreads();

  // Scaled-x form (16-bit type bf16, tensor-copy path): with one reference
  // ref for the whole tile, exp(dA_l - dA_s) dt_s = exp(dA_l - ref) *
  // (exp(ref - dA_s) dt_s).  The key factor scales the x rows of each block
  // in place, the row factor multiplies row l of D2 in the epilogue, and cb
  // feeds the MMA as loaded: only the blocks that reach the diagonal are
  // touched, to zero their keys s > l.  ref = max(lo, hi - 100) with lo the
  // smallest dA over the tile's keys and hi the largest over its rows (log2
  // units), taken when every dA / dt of those keys is finite and hi - lo <=
  // 128: then the row factor lies in [2^-28, 2^100] and the key factor
  // amplifies x dt by at most 2^28.  A key factor that underflows belongs to
  // an entry whose true decay is below 2^(100-126) for every row of the tile,
  // invisible next to the 16-bit terms of the row's own keys.  Otherwise
  // (and for fp16, whose range is too small for the scaled rows) the per-block
  // W build below.
  bool xfact = false;
  float xref = 0.0f;
  if constexpr (kTma && kBf16) {
    const float* rng = reinterpret_cast<const float*>(sm + L.rng);
    const int r0 = l0 / kSsdKBlk, r1 = min(r0 + 1, (Q - 1) / kSsdKBlk);
    const float hi = fmaxf(rng[16 + r0], rng[16 + r1]);
    float lo = rng[0];
    bool fin = rng[32] != 0.0f;
    for (int j = 1; j < nblk; ++j) {
      lo = fminf(lo, rng[j]);
      fin = fin && rng[32 + j] != 0.0f;
    }
    xfact = fin && hi - lo <= 128.0f;
    xref = fmaxf(lo, hi - 100.0f);
  }

  auto unpack2 = [](uint32_t u) -> float2 {  // a 16-bit pair -> two floats
    if constexpr (kBf16) {
      return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
    } else {
      return __half22float2(*reinterpret_cast<const __half2*>(&u));
    }
  };
  auto build_w = [&](int j) {  // cb block j -> W, in place in buffer j % 3
    const int s0 = j * kSsdKBlk, sc = s0 + cpk * 8;
    uint8_t* wb = sm + L.cbuf(j % 3);
    // exp(dA_l - dA_s) = exp(dA_l - ref) exp(ref - dA_s) with ref = dA[s0]
    // when neither factor can overflow: the block's keys lie within 2^100 of
    // ref (ref - min dA_s <= 100 in log2 units) and no row of the tile lies
    // more than 2^100 above it.  A row factor that underflows belongs to an
    // entry whose true decay exp(dA_l - dA_s) is below 2^(100-126), which is
    // invisible next to the 16-bit W of the row's own keys.  Else per entry.
    const float ref = sdA[s0];
    const float* rng = reinterpret_cast<const float*>(sm + L.rng);
    const int r0 = l0 / kSsdKBlk, r1 = min(r0 + 1, (Q - 1) / kSsdKBlk);
    const float hi_rows = fmaxf(rng[16 + r0], rng[16 + r1]);
    const bool fact = ref - rng[j] <= 100.0f && hi_rows - ref <= 100.0f;
    float2 das[4], dts[4];  // key pairs of this thread's packet
    if (sc + 8 <= Q) {  // 32-byte aligned: sc is a multiple of 8
      const float4 a0 = *reinterpret_cast<const float4*>(sdA + sc);
      const float4 a1 = *reinterpret_cast<const float4*>(sdA + sc + 4);
      const uint4 tv = *reinterpret_cast<const uint4*>(sdt + sc);  // 16-byte aligned
      das[0] = make_float2(a0.x, a0.y);
      das[1] = make_float2(a0.z, a0.w);
      das[2] = make_float2(a1.x, a1.y);
      das[3] = make_float2(a1.z, a1.w);
      dts[0] = unpack2(tv.x);
      dts[1] = unpack2(tv.y);
      dts[2] = unpack2(tv.z);
      dts[3] = unpack2(tv.w);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int s = sc + 2 * q;
        das[q] = make_float2(s < Q ? sdA[s] : ref, s + 1 < Q ? sdA[s + 1] : ref);
        dts[q] = make_float2(s < Q ? Cvt<T>::to_f(sdt[s]) : 0.0f,
                             s + 1 < Q ? Cvt<T>::to_f(sdt[s + 1]) : 0.0f);
      }
    }
    if (fact) {  // exp(ref - dA_s) dt_s
#pragma unroll
      for (int q = 0; q < 4; ++q)
        dts[q] = fmul2(dts[q], make_float2(ex2(ref - das[q].x), ex2(ref - das[q].y)));
    }
#pragma unroll
    for (int it = 0; it < kSsdRows / kSsdRowGroups; ++it) {
      const int r = rg + kSsdRowGroups * it;
      const int l = l0 + r;
      uint4* slot = reinterpret_cast<uint4*>(wb + ssd_swz(r, cpk));
      // Packets wholly above the diagonal or past the chunk are zero.
      if (!(l < Q && sc <= l && sc < Q)) {
        *slot = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      const uint4 cbv = *slot;
      const uint32_t* cw = reinterpret_cast<const uint32_t*>(&cbv);
      const float dal = sdA[l];
      // Rows whose whole packet is visible (every key <= l, < Q) skip the mask.
      const bool full = sc + 7 <= l && sc + 8 <= Q;
      const float el = fact ? ex2(dal - ref) : 0.0f;
      uint32_t pk[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 e2;
        if (fact) {
          e2 = make_float2(el, el);
        } else {
          const float2 a = fadd2(make_float2(dal, dal), make_float2(-das[q].x, -das[q].y));
          e2 = make_float2(ex2(a.x), ex2(a.y));
        }
        float2 w2 = fmul2(fmul2(unpack2(cw[q]), e2), dts[q]);
        if (!full) {
          const int s = sc + 2 * q;
          w2.x = (s <= l && s < Q) ? w2.x : 0.0f;
          w2.y = (s + 1 <= l && s + 1 < Q) ? w2.y : 0.0f;
        }
        pk[q] = pack16<T>(w2.x, w2.y);
      }
      *slot = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  };
  // Scaled-x form: x rows s of key block j times exp(ref - dA_s) dt_s, in
  // place in buffer j % 3 (64 rows of P / 8 16-byte units, the layout the
  // tensor copy wrote: 64-column chunks of [64][128 B], 128-byte swizzle).
  auto scale_x = [&](int j) {
    uint8_t* xb = sm + L.xbuf(j % 3);
    const int upr = P / 8;
    for (int i = tid; i < kSsdKBlk * upr; i += kSsdThreads) {
      const int r = static_cast<int>(p.div_x.div(i)), u = i - r * upr;
      const int s = j * kSsdKBlk + r;  // < Q: blocks never cross the chunk end here
      const float f = ex2(xref - sdA[s]) * Cvt<T>::to_f(sdt[s]);
      uint4* slot = reinterpret_cast<uint4*>(xb + (u >> 3) * (kSsdKBlk * 128) + ssd_swz(r, u & 7));
      uint4 v = *slot;
      uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 a = fmul2(unpack2(w[q]), make_float2(f, f));
        w[q] = pack16<T>(a.x, a.y);
      }
      *slot = v;
    }
  };
  // Scaled-x form, a block that reaches the diagonal: cb[l, s] -> 0 for keys
  // s > l (packets wholly above the diagonal, and the tail of the packet the
  // diagonal crosses).  Rows past the chunk arrived zero-filled.
  auto mask_cb = [&](int j) {
    const int sc = j * kSsdKBlk + cpk * 8;
    uint8_t* wb = sm + L.cbuf(j % 3);
#pragma unroll
    for (int it = 0; it < kSsdRows / kSsdRowGroups; ++it) {
      const int r = rg + kSsdRowGroups * it;
      const int l = l0 + r;
      if (sc + 7 <= l) continue;  // every key of the packet is visible
      uint4* slot = reinterpret_cast<uint4*>(wb + ssd_swz(r, cpk));
      if (sc > l) {
        *slot = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      const int keep = l - sc + 1;  // keys sc .. l stay: 1 to 7 elements
      uint4 v = *slot;
      uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // element 2q is the low half of word q
        if (2 * q >= keep) w[q] = 0u;
        else if (2 * q + 1 >= keep) w[q] &= 0x0000ffffu;
      }
      *slot = v;
    }
  };

  int issued = 0;  // key blocks whose MMAs were issued
  for (int j = 0; j < nblk; ++j) {
    // cb and x of block j landed.
    bool okj = true;
    if constexpr (kTma) {
      okj = mbar_wait(&bars->full[j % 3], (j / 3) & 1, p.err, abort_flag);
    } else if (j > 0) {  // group j: all but the groups committed after it
      if (j + 1 < nblk) cp_async_wait_prev();
      else cp_async_wait_all();
    }
    if (okj) {
      if (xfact) {
        scale_x(j);
        if (j * kSsdKBlk + kSsdKBlk - 1 > l0) mask_cb(j);
      } else {
        build_w(j);
      }
    }
    if constexpr (kTma) {
      // Buffers 1 and 2 reuse the C / prev region: blocks 1 and 2 are requested
      // once the history MMA has read it, before this iteration's barrier, so
      // a failed wait reaches every thread before any waits for block 1.
      if (j == 0 && tid == 0 && ok) {
        ok = mbar_wait(&bars->d1_done, 0, p.err, abort_flag);
        if (ok && nblk > 1) tma_blk(1);
        if (ok && nblk > 2) tma_blk(2);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    // Uniform: every thread leaves the loop here or none does.
    if (!__syncthreads_and(okj && ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 0) {
      const uint64_t a = smem_desc(sb + L.cbuf(j % 3), 16, 1024);
      const uint64_t bd = smem_desc(sb + L.xbuf(j % 3), kSsdKBlk * 128, 1024);
#pragma unroll
      for (int kk = 0; kk < kSsdKBlk / 16; ++kk)
        mma_f16_ss(t_d2, desc_advance(a, kk * 32), desc_advance(bd, kk * 16 * 128), id_kmn,
                   (j > 0 || kk > 0) ? 1u : 0u);
      mma_commit(&bars->blk_done[j % 3]);
    }
    issued = j + 1;
    if (j + 2 < nblk) {
      // Block j + 2 goes to the buffers block j - 1 read (for j = 0: the
      // third cb buffer, the C tile, which the history MMA read; on the
      // tensor-copy path block 2 was requested with block 1 above).
      if constexpr (kTma) {
        if (tid == 0 && j >= 1) {
          // A failed wait shows at the next iteration's barrier, before any
          // thread waits for the block not issued here.
          ok = mbar_wait(&bars->blk_done[(j - 1) % 3], ((j - 1) / 3) & 1, p.err, abort_flag);
          if (ok) tma_blk(j + 2);
        }
      } else {
        bool free_ok = j >= 1 ? mbar_wait(&bars->blk_done[(j - 1) % 3], ((j - 1) / 3) & 1,
                                          p.err, abort_flag)
                              : mbar_wait(&bars->d1_done, 0, p.err, abort_flag);
        if (!__syncthreads_and(free_ok)) {
          ok = false;
          break;
        }
        issue_x(j + 2);
        issue_cb(j + 2);
        cp_async_commit();
      }
    }
  }
  if constexpr (kTma) {
    // No tensor copy may still write this CTA's shared memory at exit: the
    // last block each buffer was armed for, and the C tile.
    if (tid == 0) {
      mbar_wait(&bars->c_full, 0, p.err, abort_flag, true);
      for (int i = 0; i < 3; ++i)
        if (armed[i] >= 0) mbar_wait(&bars->full[i], (armed[i] / 3) & 1, p.err, abort_flag, true);
    }
  }
  cp_async_wait_all();  // no copy may still write this CTA's shared memory at exit
  if (tid == 0) mma_commit(&bars->all_done);
  // All threads wait for the accumulators (with a failed run: for the MMAs
  // already issued, so TMEM is not freed under them).
  const bool done = mbar_wait(&bars->all_done, 0, p.err, abort_flag, !ok);
  tc_fence_after();
  // Uniform across the CTA: the epilogue below synchronises.
  if (__syncthreads_and(ok && done && issued == nblk)) {
    // out = exp(dA_l) D1 + D2, row r = TMEM lane r, staged in the freed W / x
    // buffers as fp32 rows of P (16-byte units swizzled within groups of 8
    // or 4), then written by consecutive threads along each row.
    // Warps w and w + 4 share TMEM lanes 32 (w % 4).. and take alternate
    // 32-column chunks.
    const int r = (warp & 3) * 32 + (tid & 31);
    const int l = l0 + r;
    const uint32_t lane = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float eh = l < Q ? ex2(sdA[l]) : 0.0f;
    // Scaled-x form: D2 row l still carries exp(ref - dA_s) for its keys.
    const float rfl = (xfact && l < Q) ? ex2(sdA[l] - xref) : 1.0f;
    const int U = P / 4;                            // units per row
    if (kTma && Q % kSsdRows == 0) {
      // Staged as 32-column (128-byte) slabs [128 rows][32] fp32 with the
      // 128-byte swizzle (16-byte unit u of row r at u ^ (r % 8)), each slab
      // written by one tensor store.
      uint8_t* stg = sm + L.stage();
      for (int c0 = 32 * (warp >> 2); c0 < P; c0 += 64) {
        uint32_t x1[32], x2[32];
        tmem_ld32(t_d1 + lane + c0, x1);
        tmem_ld32(t_d2 + lane + c0, x2);
        tmem_wait_ld_regs(x1);
        tmem_wait_ld_regs(x2);
        uint8_t* slab = stg + (c0 >> 5) * (kSsdRows * 128) + r * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<float4*>(slab + ((u ^ (r & 7)) << 4)) =
              make_float4(fmaf(eh, __uint_as_float(x1[4 * u]), rfl * __uint_as_float(x2[4 * u])),
                          fmaf(eh, __uint_as_float(x1[4 * u + 1]), rfl * __uint_as_float(x2[4 * u + 1])),
                          fmaf(eh, __uint_as_float(x1[4 * u + 2]), rfl * __uint_as_float(x2[4 * u + 2])),
                          fmaf(eh, __uint_as_float(x1[4 * u + 3]), rfl * __uint_as_float(x2[4 * u + 3])));
      }
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) {
        for (int c0 = 0; c0 < P; c0 += 32)
          tma_store_4d(&tm_out, stg + (c0 >> 5) * (kSsdRows * 128), c0, h, c * Q + l0, b);
        bulk_commit();
        bulk_wait_read_all();  // the staging tile is read before the CTA exits
      }
    } else {
    const int smask = (U & 7) == 0 ? 7 : 3;
    float* stg = reinterpret_cast<float*>(sm + L.stage());
    for (int c0 = 32 * (warp >> 2); c0 < P; c0 += 64) {
      uint32_t x1[32], x2[32];
      tmem_ld32(t_d1 + lane + c0, x1);
      tmem_ld32(t_d2 + lane + c0, x2);
      tmem_wait_ld_regs(x1);
      tmem_wait_ld_regs(x2);
      const int ncol = min(32, P - c0);
      for (int i = 0; i < ncol; i += 4) {
        const int u = (c0 + i) >> 2;
        const int us = (u & ~smask) | ((u ^ r) & smask);
        *reinterpret_cast<float4*>(stg + r * P + us * 4) =
            make_float4(fmaf(eh, __uint_as_float(x1[i]), rfl * __uint_as_float(x2[i])),
                        fmaf(eh, __uint_as_float(x1[i + 1]), rfl * __uint_as_float(x2[i + 1])),
                        fmaf(eh, __uint_as_float(x1[i + 2]), rfl * __uint_as_float(x2[i + 2])),
                        fmaf(eh, __uint_as_float(x1[i + 3]), rfl * __uint_as_float(x2[i + 3])));
      }
    }
    __syncthreads();
    const int rows = min(kSsdRows, Q - l0);
    for (int i = tid; i < rows * U; i += kSsdThreads) {
      const int rr = static_cast<int>(p.div_o.div(i)), u = i - rr * U;
      const int us = (u & ~smask) | ((u ^ rr) & smask);
      const float4 v = *reinterpret_cast<const float4*>(stg + rr * P + us * 4);
      __stcs(reinterpret_cast<float4*>(
                 p.out + ((static_cast<int64_t>(b) * S + c * Q + l0 + rr) * p.H + h) * P + u * 4),
             v);
    }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

template <typename T>
int launch_ssd(const SsdParams& p, cudaStream_t s) {
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  // Tensor copies need whole 64-element boxes of x / C columns and whole
  // 64-key blocks of the chunk (a block never crosses into the next chunk).
  CUtensorMap tm_x, tm_c, tm_cb, tm_out;
  memset(&tm_x, 0, sizeof(tm_x));
  memset(&tm_c, 0, sizeof(tm_c));
  memset(&tm_cb, 0, sizeof(tm_cb));
  memset(&tm_out, 0, sizeof(tm_out));
  bool tma = p.Q % 64 == 0 && p.P % 64 == 0 && p.N % 64 == 0;
  if (tma) {
    const int S = p.NC * p.Q;
    const uint64_t cb_dims[3] = {static_cast<uint64_t>(p.Q), static_cast<uint64_t>(p.Q),
                                 static_cast<uint64_t>(p.B) * p.NC * p.G};
    const uint64_t cb_strides[2] = {static_cast<uint64_t>(p.Q) * 2,
                                    static_cast<uint64_t>(p.Q) * p.Q * 2};
    const uint32_t cb_box[3] = {64, static_cast<uint32_t>(kSsdRows), 1};
    tma = make_bshd_map(&tm_x, p.x, p.P, p.H, S, p.B, kSsdKBlk, bf16) &&
          make_bshd_map(&tm_c, p.C, p.N, p.G, S, p.B, kSsdRows, bf16) &&
          make_tiled_map_16bit(&tm_cb, p.cb, bf16, 3, cb_dims, cb_strides, cb_box);
    if (tma && p.Q % kSsdRows == 0) {  // out (B, S, H, P) fp32: box (32, 1, 128, 1)
      auto fn = tensor_map_encoder();
      const cuuint64_t dims[4] = {static_cast<cuuint64_t>(p.P), static_cast<cuuint64_t>(p.H),
                                  static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(p.B)};
      const cuuint64_t strides[3] = {static_cast<cuuint64_t>(p.P) * 4,
                                     static_cast<cuuint64_t>(p.P) * p.H * 4,
                                     static_cast<cuuint64_t>(p.P) * p.H * S * 4};
      const cuuint32_t box[4] = {32, 1, static_cast<cuuint32_t>(kSsdRows), 1};
      const cuuint32_t estride[4] = {1, 1, 1, 1};
      tma = fn && fn(&tm_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.out, dims, strides, box,
                     estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
  }
  auto k = tma ? ssd_chunk_scan<T, true> : ssd_chunk_scan<T, false>;
  const int smem = SsdLayout(p.P, p.N, p.Q, tma).bytes + 1024;  // + room to align the base
  if (smem > 232448) return TILEOPS_EBADSHAPE;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return TILEOPS_ELAUNCH;
  const int64_t grid = static_cast<int64_t>(p.B) * p.NC * p.H * p.ltiles;
  k<<<static_cast<unsigned>(grid), kSsdThreads, smem, s>>>(p, tm_x, tm_c, tm_cb, tm_out);
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
  p.div_c = FastDivU32(static_cast<uint32_t>(((d_state + 15) & ~15) / 8));
  p.div_x = FastDivU32(static_cast<uint32_t>(d_head / 8));
  p.div_o = FastDivU32(static_cast<uint32_t>(d_head / 4));
  p.err = device_error_ptr();
  cudaStream_t s = as_stream(stream);
  return dtype == TILEOPS_DT_BF16 ? launch_ssd<__nv_bfloat16>(p, s) : launch_ssd<__half>(p, s);
}
