// sbda_kernels.cu -- SBDA sparse gather-softmax attention for B200 (sm_100a).
//
// Forward and gather-form backward of the exact-source attention that the
// reference implements in Triton (BiAttn/sbda_triton.py:134-201 block forward,
// :440-503 weights, :506-587 dQ, :590-671 key-centric dK/dV) and in eager
// PyTorch (BiAttn/left_v2.py:335-405).
//
// Design (B200-first, not a translation of the Triton kernels):
//  * The path is a 4-way gather (about 1.5 flop per byte), so it is bound by
//    HBM bandwidth and uses no tensor cores.
//  * One CTA owns a tile of TILE consecutive positions of one (batch, head).
//    Its rows are staged in shared memory by TMA (cp.async.bulk.tensor, no
//    multicast) from 4-D tensor maps over the caller's strided [B,H,L,D]
//    view.  Rows before position 0 or past L are zero-filled by the copy
//    engine; scores are still masked explicitly (i - o >= 0).
//  * Offsets are split into a "near" window (o <= TILE: one contiguous tile
//    with a left halo of Hn rows) and at most one "far" (dyadic) offset f
//    with its own tile.  When f is a multiple of TILE the tiles are launched
//    in chain order t, t+f/TILE, t+2f/TILE, ... so the far tile a CTA reads is
//    the tile the previous CTA in launch order read as its own: it is an L2
//    hit, and every K/V byte crosses HBM about once per pass.
//  * Eight lanes own one row (16-byte vectors; a row pitch of 128*NV bytes
//    holds D padded with zeros by the copy engine), the 4 dot products are
//    reduced with xor-shuffles, the softmax runs in fp32 registers.
//  * The forward writes O (input dtype) and a fp32 log-sum-exp per row.
//  * The backward is gather form and atomic-free: the CTA of key tile
//    [j0, j0+TILE) recomputes the softmax of every consumer query of its keys
//    ([j0, j0+TILE+Hn) and [j0+f, j0+f+TILE)), writes dQ for its own queries
//    and dK/dV for its own keys, each exactly once.  Native GQA: the CTA owns
//    a kv head and loops over the H/kv_heads query heads that share it.
//  * Every wait on a copy barrier is bounded; on expiry the kernel sets a
//    device fault word (read by sbda_b200_device_status) and returns.

#include "sbda_b200.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <math.h>
#include <mutex>
#include <stdint.h>
#include <string.h>

namespace sbda {

constexpr int kThreads = 128;             // 4 warps
constexpr int kGroups = kThreads / 8;     // 8-lane row groups per CTA
constexpr unsigned kFaultWaitExpired = 1u;

__device__ unsigned int g_device_status = 0;

// --------------------------------------------------------------------------
// Kernel parameters
// --------------------------------------------------------------------------

struct TensorArg {
  const void* ptr;
  long long sb, sh, sl, sd;  // element strides
};

struct Geometry {
  int S;           // number of sources (1..4)
  int off[4];      // offsets
  int is_far[4];   // 1 for the far source
  int Hn;          // near halo rows = largest near offset
  int f;           // far offset (0 if none)
  int has_far;
  int nT;          // tiles per (batch, head)
  int R, A, rem;   // chain order: R = f / TILE tiles per chain step (0 = linear)
};

struct FwdParams {
  int B, H, Hkv, G, L, D;
  float scale;
  Geometry g;
  TensorArg q, k, v, out;
  float* lse;
  unsigned slots_q, slots_k, slots_v;
};

struct BwdParams {
  int B, H, Hkv, G, L, D;
  float scale;
  Geometry g;
  TensorArg q, k, v, dout, dq, dk, dv;
  const float* lse;
  unsigned slots_q, slots_k, slots_v, slots_d;
};

// Tensor maps: *T = TILE-row box, *H = Hn-row halo box.
struct FwdMaps {
  CUtensorMap qT, kT, vT, kH, vH;
};
struct BwdMaps {
  CUtensorMap qT, qH, dT, dH, kT, kH, vT, vH;
};

// --------------------------------------------------------------------------
// Device helpers: mbarrier + TMA (inline PTX), element packing
// --------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the barrier phase with a 2 s bound.  Returns false on expiry.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - start > 2000000000ull) return false;
  }
}

// Records a device fault, waits once more (bounded) for copies still in
// flight into this CTA's shared memory, and lets the caller return.
__device__ __forceinline__ void fault_and_drain(uint64_t* bar, uint32_t parity) {
  if (threadIdx.x == 0) atomicOr(&g_device_status, kFaultWaitExpired);
  (void)mbar_wait_bounded(bar, parity);
}

// 4-D tiled TMA load; coordinate 0 is the channel (always 0, so the 16-byte
// rule on the innermost coordinate holds), slots say where position / head /
// batch sit among coordinates 1..3 of this tensor's map.
__device__ __forceinline__ void tma_rows(void* dst, const CUtensorMap* map, uint64_t* bar, unsigned slots,
                                         int pos, int head, int batch) {
  const int sl = slots & 3, sh = (slots >> 2) & 3;
  const int c1 = sl == 1 ? pos : (sh == 1 ? head : batch);
  const int c2 = sl == 2 ? pos : (sh == 2 ? head : batch);
  const int c3 = sl == 3 ? pos : (sh == 3 ? head : batch);
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

template <typename TE>
struct Elem;
template <>
struct Elem<float> {
  static __device__ __forceinline__ void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
  static __device__ __forceinline__ float to_float(float x) { return x; }
  static __device__ __forceinline__ float from_float(float x) { return x; }
};
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ void unpack2(uint32_t w, float* f) {
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xffff0000u);
  }
  static __device__ __forceinline__ void unpack(const uint4& u, float* f) {
    unpack2(u.x, f);
    unpack2(u.y, f + 2);
    unpack2(u.z, f + 4);
    unpack2(u.w, f + 6);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
  static __device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Elem<__half> {
  static __device__ __forceinline__ void unpack2(uint32_t w, float* f) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w));
    f[0] = t.x;
    f[1] = t.y;
  }
  static __device__ __forceinline__ void unpack(const uint4& u, float* f) {
    unpack2(u.x, f);
    unpack2(u.y, f + 2);
    unpack2(u.z, f + 4);
    unpack2(u.w, f + 6);
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
  static __device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_float(float x) { return __float2half_rn(x); }
};

// Row of a staged tile -> this lane's EPL floats.  Lane l8 of the row group
// owns 16-byte vectors l8, l8+8, l8+16, ...
template <typename TE, int NV>
__device__ __forceinline__ void load_row(const uint8_t* row, int l8, float* f) {
  constexpr int VE = 16 / sizeof(TE);
#pragma unroll
  for (int n = 0; n < NV; ++n) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + (l8 + 8 * n) * 16);
    Elem<TE>::unpack(u, f + n * VE);
  }
}

template <typename TE, int NV, bool VEC>
__device__ __forceinline__ void store_row(TE* dst, long long sd, int D, int l8, const float* f) {
  constexpr int VE = 16 / sizeof(TE);
#pragma unroll
  for (int n = 0; n < NV; ++n) {
    const int c0 = (l8 + 8 * n) * VE;
    if (c0 >= D) continue;
    if constexpr (VEC) {
      *reinterpret_cast<uint4*>(dst + c0) = Elem<TE>::pack(f + n * VE);
    } else {
#pragma unroll
      for (int e = 0; e < VE; ++e)
        if (c0 + e < D) dst[(long long)(c0 + e) * sd] = Elem<TE>::from_float(f[n * VE + e]);
    }
  }
}

// Cooperative zero-filling load of rows [pos0, pos0 + rows) of one
// (batch, head) slice into a staged tile (pitch = pitch_elems elements).
// Used when a tensor's layout does not meet the copy engine's alignment rules.
template <typename TE>
__device__ void generic_rows(uint8_t* dst, const TensorArg& t, int batch, int head, int pos0, int rows, int L,
                             int D, int pitch_elems) {
  TE* out = reinterpret_cast<TE*>(dst);
  const TE* src = reinterpret_cast<const TE*>(t.ptr);
  const int total = rows * pitch_elems;
  for (int e = threadIdx.x; e < total; e += blockDim.x) {
    const int r = e / pitch_elems, c = e - r * pitch_elems;
    const long long pos = (long long)pos0 + r;
    TE val = Elem<TE>::from_float(0.f);
    if (c < D && pos >= 0 && pos < L)
      val = src[(long long)batch * t.sb + (long long)head * t.sh + pos * t.sl + (long long)c * t.sd];
    out[e] = val;
  }
}

__device__ __forceinline__ int chain_tile(int idx, const Geometry& g) {
  if (g.R == 0) return idx;
  const int full = g.rem * g.A;
  int r, a;
  if (idx < full) {
    r = idx / g.A;
    a = idx - r * g.A;
  } else {
    const int j = idx - full, a1 = g.A - 1;
    r = g.rem + j / a1;
    a = j - (j / a1) * a1;
  }
  return a * g.R + r;
}

template <int EPL>
__device__ __forceinline__ float dot(const float* a, const float* b) {
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc = fmaf(a[e], b[e], acc);
  return acc;
}

__device__ __forceinline__ float group_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  return x;
}

// --------------------------------------------------------------------------
// Forward
// --------------------------------------------------------------------------

template <typename TE, int NV, int TILE, bool TMA>
__global__ void __launch_bounds__(kThreads) sbda_fwd_kernel(const __grid_constant__ FwdMaps maps,
                                                            const FwdParams p) {
  constexpr int VE = 16 / sizeof(TE);
  constexpr int EPL = NV * VE;
  constexpr int P = NV * 128;  // staged row pitch (bytes)
  extern __shared__ __align__(128) uint8_t smem[];
  const Geometry& g = p.g;
  const int tid = threadIdx.x, lane = tid & 31;
  const int grp = (tid >> 5) * 4 + (lane >> 3), l8 = lane & 7;

  int bid = blockIdx.x;
  const int h = bid % p.H;
  bid /= p.H;
  const int t = chain_tile(bid % g.nT, g);
  const int b = bid / g.nT;
  const int hk = h / p.G;
  const int i0 = t * TILE;
  const int Hn = g.Hn;

  uint8_t* Qs = smem;
  uint8_t* Kn = Qs + TILE * P;
  uint8_t* Vn = Kn + (Hn + TILE) * P;
  uint8_t* Kf = Vn + (Hn + TILE) * P;
  uint8_t* Vf = Kf + (g.has_far ? TILE * P : 0);
  uint64_t* bar = reinterpret_cast<uint64_t*>(Vf + (g.has_far ? TILE * P : 0));

  if constexpr (TMA) {
    if (tid == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
      const uint32_t bytes = (uint32_t)((TILE * (3 + 2 * g.has_far) + 2 * Hn) * P);
      mbar_arrive_expect_tx(bar, bytes);
      tma_rows(Qs, &maps.qT, bar, p.slots_q, i0, h, b);
      if (Hn > 0) {
        tma_rows(Kn, &maps.kH, bar, p.slots_k, i0 - Hn, hk, b);
        tma_rows(Vn, &maps.vH, bar, p.slots_v, i0 - Hn, hk, b);
      }
      tma_rows(Kn + Hn * P, &maps.kT, bar, p.slots_k, i0, hk, b);
      tma_rows(Vn + Hn * P, &maps.vT, bar, p.slots_v, i0, hk, b);
      if (g.has_far) {
        tma_rows(Kf, &maps.kT, bar, p.slots_k, i0 - g.f, hk, b);
        tma_rows(Vf, &maps.vT, bar, p.slots_v, i0 - g.f, hk, b);
      }
    }
    const bool ok = mbar_wait_bounded(bar, 0);
    if (__syncthreads_or(!ok)) {
      fault_and_drain(bar, 0);
      return;
    }
  } else {
    constexpr int PE = P / sizeof(TE);
    generic_rows<TE>(Qs, p.q, b, h, i0, TILE, p.L, p.D, PE);
    generic_rows<TE>(Kn, p.k, b, hk, i0 - Hn, Hn + TILE, p.L, p.D, PE);
    generic_rows<TE>(Vn, p.v, b, hk, i0 - Hn, Hn + TILE, p.L, p.D, PE);
    if (g.has_far) {
      generic_rows<TE>(Kf, p.k, b, hk, i0 - g.f, TILE, p.L, p.D, PE);
      generic_rows<TE>(Vf, p.v, b, hk, i0 - g.f, TILE, p.L, p.D, PE);
    }
    __syncthreads();
  }

  const float scale = p.scale;
  TE* out = reinterpret_cast<TE*>(const_cast<void*>(p.out.ptr));
  float* lse = p.lse + ((long long)b * p.H + h) * p.L;
#pragma unroll 1
  for (int r = grp; r < TILE; r += kGroups) {
    const int i = i0 + r;
    float qf[EPL];
    load_row<TE, NV>(Qs + r * P, l8, qf);
    float sc[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      sc[s] = 0.f;
      if (s < g.S) {
        const uint8_t* kr = g.is_far[s] ? Kf + r * P : Kn + (Hn + r - g.off[s]) * P;
        float kf[EPL];
        load_row<TE, NV>(kr, l8, kf);
        sc[s] = group_sum(dot<EPL>(qf, kf));
      }
    }
    float mx = -INFINITY;
    bool valid[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      valid[s] = s < g.S && i - g.off[s] >= 0;
      sc[s] = valid[s] ? sc[s] * scale : -INFINITY;
      mx = fmaxf(mx, sc[s]);
    }
    float pr[4], sum = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      pr[s] = valid[s] ? __expf(sc[s] - mx) : 0.f;
      sum += pr[s];
    }
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    float of[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) of[e] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      if (s < g.S) {
        const float w = pr[s] * inv;
        const uint8_t* vr = g.is_far[s] ? Vf + r * P : Vn + (Hn + r - g.off[s]) * P;
        float vf[EPL];
        load_row<TE, NV>(vr, l8, vf);
#pragma unroll
        for (int e = 0; e < EPL; ++e) of[e] = fmaf(w, vf[e], of[e]);
      }
    }
    if (i < p.L) {
      TE* orow = out + (long long)b * p.out.sb + (long long)h * p.out.sh + (long long)i * p.out.sl;
      store_row<TE, NV, TMA>(orow, p.out.sd, p.D, l8, of);
      if (l8 == 0) lse[i] = sum > 0.f ? mx + __logf(sum) : -INFINITY;
    }
  }
}

// --------------------------------------------------------------------------
// Backward (gather form)
// --------------------------------------------------------------------------

template <typename TE, int NV, int TILE, bool TMA>
__global__ void __launch_bounds__(kThreads) sbda_bwd_kernel(const __grid_constant__ BwdMaps maps,
                                                            const BwdParams p) {
  constexpr int VE = 16 / sizeof(TE);
  constexpr int EPL = NV * VE;
  constexpr int P = NV * 128;
  constexpr int KROWS = TILE / kGroups;  // key rows per row group
  extern __shared__ __align__(128) uint8_t smem[];
  const Geometry& g = p.g;
  const int tid = threadIdx.x, lane = tid & 31;
  const int grp = (tid >> 5) * 4 + (lane >> 3), l8 = lane & 7;

  int bid = blockIdx.x;
  const int hk = bid % p.Hkv;
  bid /= p.Hkv;
  const int t = chain_tile(bid % g.nT, g);
  const int b = bid / g.nT;
  const int j0 = t * TILE;
  const int Hn = g.Hn, far = g.has_far, f = g.f;
  const int NC = TILE + Hn + (far ? TILE : 0);  // consumer rows

  // Staged regions (rows of P bytes).
  uint8_t* QN = smem;                        // Q of near consumers  [j0, j0+TILE+Hn)
  uint8_t* DN = QN + (TILE + Hn) * P;        // dO of near consumers
  uint8_t* KN = DN + (TILE + Hn) * P;        // K of near sources    [j0-Hn, j0+TILE+Hn)
  uint8_t* VN = KN + (TILE + 2 * Hn) * P;
  uint8_t* KFL = VN + (TILE + 2 * Hn) * P;   // far sources of near consumers [j0-f, j0-f+TILE+Hn)
  uint8_t* VFL = KFL + (far ? (TILE + Hn) * P : 0);
  uint8_t* QF = VFL + (far ? (TILE + Hn) * P : 0);  // far consumers [j0+f, j0+f+TILE)
  uint8_t* DF = QF + (far ? TILE * P : 0);
  uint8_t* KFR = DF + (far ? TILE * P : 0);  // near sources of far consumers [j0+f-Hn, j0+f+TILE)
  uint8_t* VFR = KFR + (far ? (Hn + TILE) * P : 0);
  float2* EDGE = reinterpret_cast<float2*>(VFR + (far ? (Hn + TILE) * P : 0));  // [NC][4] (p, dS)
  uint64_t* bar = reinterpret_cast<uint64_t*>(EDGE + NC * 4);

  if constexpr (TMA) {
    if (tid == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
    }
    __syncthreads();
  }

  float acc_k[KROWS][EPL], acc_v[KROWS][EPL];
#pragma unroll
  for (int k = 0; k < KROWS; ++k)
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc_k[k][e] = acc_v[k][e] = 0.f;

  const float scale = p.scale;
  TE* dq_base = reinterpret_cast<TE*>(p.dq.ptr ? const_cast<void*>(p.dq.ptr) : nullptr);

#pragma unroll 1
  for (int gi = 0; gi < p.G; ++gi) {
    const int h = hk * p.G + gi;
    if constexpr (TMA) {
      if (tid == 0) {
        uint32_t rows = 2 * (TILE + Hn) + (far ? 2 * TILE : 0);
        if (gi == 0) rows += 2 * (TILE + 2 * Hn) + (far ? 2 * (TILE + Hn) + 2 * (Hn + TILE) : 0);
        mbar_arrive_expect_tx(bar, rows * P);
        tma_rows(QN, &maps.qT, bar, p.slots_q, j0, h, b);
        tma_rows(DN, &maps.dT, bar, p.slots_d, j0, h, b);
        if (Hn > 0) {
          tma_rows(QN + TILE * P, &maps.qH, bar, p.slots_q, j0 + TILE, h, b);
          tma_rows(DN + TILE * P, &maps.dH, bar, p.slots_d, j0 + TILE, h, b);
        }
        if (far) {
          tma_rows(QF, &maps.qT, bar, p.slots_q, j0 + f, h, b);
          tma_rows(DF, &maps.dT, bar, p.slots_d, j0 + f, h, b);
        }
        if (gi == 0) {
          tma_rows(KN + Hn * P, &maps.kT, bar, p.slots_k, j0, hk, b);
          tma_rows(VN + Hn * P, &maps.vT, bar, p.slots_v, j0, hk, b);
          if (Hn > 0) {
            tma_rows(KN, &maps.kH, bar, p.slots_k, j0 - Hn, hk, b);
            tma_rows(VN, &maps.vH, bar, p.slots_v, j0 - Hn, hk, b);
            tma_rows(KN + (Hn + TILE) * P, &maps.kH, bar, p.slots_k, j0 + TILE, hk, b);
            tma_rows(VN + (Hn + TILE) * P, &maps.vH, bar, p.slots_v, j0 + TILE, hk, b);
          }
          if (far) {
            tma_rows(KFL, &maps.kT, bar, p.slots_k, j0 - f, hk, b);
            tma_rows(VFL, &maps.vT, bar, p.slots_v, j0 - f, hk, b);
            tma_rows(KFR + Hn * P, &maps.kT, bar, p.slots_k, j0 + f, hk, b);
            tma_rows(VFR + Hn * P, &maps.vT, bar, p.slots_v, j0 + f, hk, b);
            if (Hn > 0) {
              tma_rows(KFL + TILE * P, &maps.kH, bar, p.slots_k, j0 - f + TILE, hk, b);
              tma_rows(VFL + TILE * P, &maps.vH, bar, p.slots_v, j0 - f + TILE, hk, b);
              tma_rows(KFR, &maps.kH, bar, p.slots_k, j0 + f - Hn, hk, b);
              tma_rows(VFR, &maps.vH, bar, p.slots_v, j0 + f - Hn, hk, b);
            }
          }
        }
      }
      const bool ok = mbar_wait_bounded(bar, gi & 1);
      if (__syncthreads_or(!ok)) {
        fault_and_drain(bar, gi & 1);
        return;
      }
    } else {
      constexpr int PE = P / sizeof(TE);
      generic_rows<TE>(QN, p.q, b, h, j0, TILE + Hn, p.L, p.D, PE);
      generic_rows<TE>(DN, p.dout, b, h, j0, TILE + Hn, p.L, p.D, PE);
      if (far) {
        generic_rows<TE>(QF, p.q, b, h, j0 + f, TILE, p.L, p.D, PE);
        generic_rows<TE>(DF, p.dout, b, h, j0 + f, TILE, p.L, p.D, PE);
      }
      if (gi == 0) {
        generic_rows<TE>(KN, p.k, b, hk, j0 - Hn, TILE + 2 * Hn, p.L, p.D, PE);
        generic_rows<TE>(VN, p.v, b, hk, j0 - Hn, TILE + 2 * Hn, p.L, p.D, PE);
        if (far) {
          generic_rows<TE>(KFL, p.k, b, hk, j0 - f, TILE + Hn, p.L, p.D, PE);
          generic_rows<TE>(VFL, p.v, b, hk, j0 - f, TILE + Hn, p.L, p.D, PE);
          generic_rows<TE>(KFR, p.k, b, hk, j0 + f - Hn, Hn + TILE, p.L, p.D, PE);
          generic_rows<TE>(VFR, p.v, b, hk, j0 + f - Hn, Hn + TILE, p.L, p.D, PE);
        }
      }
      __syncthreads();
    }

    // ---- Phase 1: softmax of every consumer query; dQ of own queries. ----
    const float* lse = p.lse + ((long long)b * p.H + h) * p.L;
#pragma unroll 1
    for (int base = 0; base < NC; base += kGroups) {
      const bool act = base + grp < NC;
      const int c = act ? base + grp : NC - 1;
      const bool nearc = c < TILE + Hn;
      const int cf = c - (TILE + Hn);
      const int q = nearc ? j0 + c : j0 + f + cf;
      const bool inr = q < p.L;
      const float lq = inr ? lse[q] : 0.f;
      float qf[EPL], df[EPL];
      load_row<TE, NV>(nearc ? QN + c * P : QF + cf * P, l8, qf);
      load_row<TE, NV>(nearc ? DN + c * P : DF + cf * P, l8, df);
      float pr[4], dp[4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        pr[s] = 0.f;
        dp[s] = 0.f;
        if (s < g.S) {
          const uint8_t *kr, *vr;
          if (g.is_far[s]) {
            kr = nearc ? KFL + c * P : KN + (Hn + cf) * P;
            vr = nearc ? VFL + c * P : VN + (Hn + cf) * P;
          } else {
            const int rr = (nearc ? c : cf) + Hn - g.off[s];
            kr = (nearc ? KN : KFR) + rr * P;
            vr = (nearc ? VN : VFR) + rr * P;
          }
          float kf[EPL], vf[EPL];
          load_row<TE, NV>(kr, l8, kf);
          load_row<TE, NV>(vr, l8, vf);
          pr[s] = group_sum(dot<EPL>(qf, kf));
          dp[s] = group_sum(dot<EPL>(df, vf));
        }
      }
      float delta = 0.f;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const bool valid = s < g.S && inr && q - g.off[s] >= 0;
        pr[s] = valid ? __expf(fmaf(pr[s], scale, -lq)) : 0.f;
        delta = fmaf(pr[s], dp[s], delta);
      }
      float ds[4];
#pragma unroll
      for (int s = 0; s < 4; ++s) ds[s] = pr[s] * (dp[s] - delta);

      if (nearc && c < TILE && inr && act && dq_base) {
        float gq[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) gq[e] = 0.f;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          if (s < g.S) {
            const uint8_t* kr = g.is_far[s] ? KFL + c * P : KN + (c + Hn - g.off[s]) * P;
            float kf[EPL];
            load_row<TE, NV>(kr, l8, kf);
            const float w = ds[s] * scale;
#pragma unroll
            for (int e = 0; e < EPL; ++e) gq[e] = fmaf(w, kf[e], gq[e]);
          }
        }
        TE* dst = dq_base + (long long)b * p.dq.sb + (long long)h * p.dq.sh + (long long)q * p.dq.sl;
        store_row<TE, NV, TMA>(dst, p.dq.sd, p.D, l8, gq);
      }
      if (act && l8 < 4) {
        const float pv = l8 == 0 ? pr[0] : l8 == 1 ? pr[1] : l8 == 2 ? pr[2] : pr[3];
        const float dv = l8 == 0 ? ds[0] : l8 == 1 ? ds[1] : l8 == 2 ? ds[2] : ds[3];
        EDGE[c * 4 + l8] = make_float2(pv, dv);
      }
    }
    __syncthreads();

    // ---- Phase 2: gather dK / dV of own keys from their consumers. ----
#pragma unroll
    for (int k = 0; k < KROWS; ++k) {
      const int r = grp + k * kGroups;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        if (s < g.S) {
          int c;
          const uint8_t *qr, *dr;
          if (g.is_far[s]) {
            c = TILE + Hn + r;
            qr = QF + r * P;
            dr = DF + r * P;
          } else {
            c = r + g.off[s];
            qr = QN + c * P;
            dr = DN + c * P;
          }
          const float2 e2 = EDGE[c * 4 + s];
          float qf[EPL], df[EPL];
          load_row<TE, NV>(qr, l8, qf);
          load_row<TE, NV>(dr, l8, df);
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            acc_k[k][e] = fmaf(e2.y, qf[e], acc_k[k][e]);
            acc_v[k][e] = fmaf(e2.x, df[e], acc_v[k][e]);
          }
        }
      }
    }
    __syncthreads();  // staged Q/dO and EDGE are rewritten by the next query head
  }

  TE* dk = reinterpret_cast<TE*>(const_cast<void*>(p.dk.ptr));
  TE* dv = reinterpret_cast<TE*>(const_cast<void*>(p.dv.ptr));
#pragma unroll
  for (int k = 0; k < KROWS; ++k) {
    const int j = j0 + grp + k * kGroups;
    if (j >= p.L) continue;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc_k[k][e] *= scale;
    store_row<TE, NV, TMA>(dk + (long long)b * p.dk.sb + (long long)hk * p.dk.sh + (long long)j * p.dk.sl,
                           p.dk.sd, p.D, l8, acc_k[k]);
    store_row<TE, NV, TMA>(dv + (long long)b * p.dv.sb + (long long)hk * p.dv.sh + (long long)j * p.dv.sl,
                           p.dv.sd, p.D, l8, acc_v[k]);
  }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

int elem_size(int dtype) { return dtype == SBDA_DTYPE_F32 ? 4 : 2; }

CUtensorMapDataType map_dtype(int dtype) {
  return dtype == SBDA_DTYPE_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
         : dtype == SBDA_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// Row pitch of a staged tile: D padded to a power of two, at least 128 bytes.
int row_pitch(int64_t D, int e) {
  int p = 128;
  while (p < D * e) p *= 2;
  return p;
}

struct View {
  const void* ptr;
  int64_t heads;
  sbda_tensor t;
};

// A view can be staged by the copy engine / written with 16-byte vectors when
// its base and the byte strides of every non-trivial outer dimension are
// multiples of 16 and channels are contiguous.
bool vector_ok(const sbda_tensor& t, int64_t B, int64_t H, int64_t L, int64_t D, int e) {
  if (reinterpret_cast<uintptr_t>(t.data) % 16) return false;
  if (D > 1 && t.stride_d != 1) return false;
  if ((D * e) % 16) return false;
  const int64_t sizes[3] = {B, H, L};
  const int64_t strides[3] = {t.stride_b, t.stride_h, t.stride_l};
  for (int i = 0; i < 3; ++i)
    if (sizes[i] > 1 && (strides[i] <= 0 || (strides[i] * e) % 16)) return false;
  return true;
}

// Encodes the (D, outer...) 4-D map of a view with a box of `rows` positions.
// Outer dimensions are ordered by increasing stride; `slots` records where
// position / head / batch land (2 bits each).
bool encode_map(CUtensorMap* map, unsigned* slots, const sbda_tensor& t, int dtype, int64_t B, int64_t H,
                int64_t L, int64_t D, int pitch, int rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const int e = elem_size(dtype);
  int64_t size[3] = {L, H, B};
  int64_t stride[3] = {t.stride_l * e, t.stride_h * e, t.stride_b * e};
  int64_t big = 16;
  for (int i = 0; i < 3; ++i)
    if (size[i] > 1) big = (stride[i] * size[i] > big) ? stride[i] * size[i] : big;
  for (int i = 0; i < 3; ++i)
    if (size[i] <= 1) stride[i] = ((big + 15) / 16) * 16;  // trivial dims go outermost
  int order[3] = {0, 1, 2};
  for (int a = 0; a < 3; ++a)
    for (int c = a + 1; c < 3; ++c)
      if (stride[order[c]] < stride[order[a]]) {
        const int tmp = order[a];
        order[a] = order[c];
        order[c] = tmp;
      }
  cuuint64_t gdim[4] = {(cuuint64_t)D, 0, 0, 0};
  cuuint64_t gstride[3];
  cuuint32_t box[4] = {(cuuint32_t)(pitch / e), 1, 1, 1};
  cuuint32_t estride[4] = {1, 1, 1, 1};
  unsigned s = 0;
  for (int k = 0; k < 3; ++k) {
    const int d = order[k];
    gdim[k + 1] = (cuuint64_t)size[d];
    gstride[k] = (cuuint64_t)stride[d];
    if (d == 0) {
      box[k + 1] = (cuuint32_t)rows;
      s |= (unsigned)(k + 1);
    } else if (d == 1) {
      s |= (unsigned)(k + 1) << 2;
    } else {
      s |= (unsigned)(k + 1) << 4;
    }
  }
  *slots = s;
  const CUresult r = enc(map, map_dtype(dtype), 4, const_cast<void*>(t.data), gdim, gstride, box, estride,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct Plan {
  int tile;
  int nv;
  int pitch;
  Geometry g;
  size_t smem_fwd, smem_bwd;
};

// Splits offsets into the near window and at most one far offset for a tile
// height, and sizes the staged regions.  Returns false when the offsets need
// two far tiles at this tile height.
bool plan_for_tile(const int32_t* off, int n, int64_t L, int tile, int pitch, Plan* pl) {
  Geometry g;
  memset(&g, 0, sizeof(g));
  g.S = n;
  int nfar = 0;
  for (int s = 0; s < n; ++s) {
    g.off[s] = off[s];
    if (off[s] > tile) {
      g.is_far[s] = 1;
      g.f = off[s];
      ++nfar;
    } else if (off[s] > g.Hn) {
      g.Hn = off[s];
    }
  }
  if (nfar > 1) return false;
  g.has_far = nfar;
  g.nT = (int)((L + tile - 1) / tile);
  g.R = g.A = g.rem = 0;
  if (g.has_far && g.f % tile == 0) {
    const int R = g.f / tile;
    if (R < g.nT) {
      g.R = R;
      g.A = (g.nT + R - 1) / R;
      g.rem = g.nT - (g.A - 1) * R;
    }
  }
  const size_t P = pitch;
  const size_t T = tile, Hn = g.Hn, F = g.has_far;
  pl->tile = tile;
  pl->pitch = pitch;
  pl->nv = pitch / 128;
  pl->g = g;
  pl->smem_fwd = (T + 2 * (Hn + T) + 2 * T * F) * P + 16;
  const size_t nc = T + Hn + F * T;
  pl->smem_bwd = (2 * (T + Hn) + 2 * (T + 2 * Hn) + F * (2 * (T + Hn) + 2 * T + 2 * (Hn + T))) * P +
                 nc * 4 * sizeof(float2) + 16;
  return true;
}

constexpr size_t kMaxSmem = 227 * 1024;

int make_plan(const int32_t* off, int n, int64_t L, int64_t D, int e, Plan* pl) {
  const int pitch = row_pitch(D, e);
  const int nv = pitch / 128;
  const int elems = nv * (16 / e);  // floats per lane per row
  // Tile heights instantiated per pitch, largest first.  The backward keeps
  // TILE/16 * EPL * 2 fp32 key accumulators per thread; keep that <= 64.
  int tiles[2] = {64, 0};
  if (nv == 2) {
    tiles[0] = elems <= 8 ? 64 : 32;
    tiles[1] = elems <= 8 ? 32 : 0;
  } else if (nv == 4) {
    tiles[0] = 32;
    tiles[1] = 16;
  }
  for (int i = 0; i < 2 && tiles[i]; ++i) {
    Plan cand;
    if (!plan_for_tile(off, n, L, tiles[i], pitch, &cand)) continue;
    if (cand.smem_fwd > kMaxSmem || cand.smem_bwd > kMaxSmem) continue;
    *pl = cand;
    return SBDA_OK;
  }
  return SBDA_ERR_UNSUPPORTED;
}

int validate(int dtype, const sbda_shape& s, const int32_t* off, int n) {
  if (dtype != SBDA_DTYPE_F32 && dtype != SBDA_DTYPE_F16 && dtype != SBDA_DTYPE_BF16) return SBDA_ERR_DTYPE;
  if (s.batch < 0 || s.heads < 0 || s.kv_heads < 0 || s.length < 0 || s.head_dim < 1) return SBDA_ERR_INVALID;
  if (s.head_dim > 128) return SBDA_ERR_INVALID;
  if (s.kv_heads == 0 ? s.heads != 0 : s.heads % s.kv_heads) return SBDA_ERR_INVALID;
  if (s.length > (int64_t)1 << 30 || s.batch * s.heads > ((int64_t)1 << 31) / 2) return SBDA_ERR_UNSUPPORTED;
  if (!off || n < 1 || n > 4) return SBDA_ERR_INVALID;
  for (int a = 0; a < n; ++a) {
    if (off[a] < 0) return SBDA_ERR_INVALID;
    for (int c = a + 1; c < n; ++c)
      if (off[a] == off[c]) return SBDA_ERR_INVALID;
  }
  return SBDA_OK;
}

TensorArg arg_of(const sbda_tensor& t) {
  return TensorArg{t.data, t.stride_b, t.stride_h, t.stride_l, t.stride_d};
}

template <typename TE, int NV, int TILE, bool TMA>
int launch_fwd(const FwdMaps& maps, const FwdParams& p, const Plan& pl, cudaStream_t stream) {
  auto kern = sbda_fwd_kernel<TE, NV, TILE, TMA>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem_fwd) != cudaSuccess)
    return SBDA_ERR_CUDA;
  const long long blocks = (long long)p.B * p.H * pl.g.nT;
  kern<<<(unsigned)blocks, kThreads, pl.smem_fwd, stream>>>(maps, p);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE, int NV, int TILE, bool TMA>
int launch_bwd(const BwdMaps& maps, const BwdParams& p, const Plan& pl, cudaStream_t stream) {
  auto kern = sbda_bwd_kernel<TE, NV, TILE, TMA>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem_bwd) != cudaSuccess)
    return SBDA_ERR_CUDA;
  const long long blocks = (long long)p.B * p.Hkv * pl.g.nT;
  kern<<<(unsigned)blocks, kThreads, pl.smem_bwd, stream>>>(maps, p);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

// Instantiated (pitch, tile) pairs: 128 B -> 64; 256 B -> 64, 32; 512 B -> 32, 16.
#define SBDA_FOR_TILES(LAUNCH, TE, TMA, ...)                                        \
  do {                                                                              \
    if (pl.nv == 1 && pl.tile == 64) return LAUNCH<TE, 1, 64, TMA>(__VA_ARGS__);    \
    if (pl.nv == 2 && pl.tile == 64) return LAUNCH<TE, 2, 64, TMA>(__VA_ARGS__);    \
    if (pl.nv == 2 && pl.tile == 32) return LAUNCH<TE, 2, 32, TMA>(__VA_ARGS__);    \
    if (pl.nv == 4 && pl.tile == 32) return LAUNCH<TE, 4, 32, TMA>(__VA_ARGS__);    \
    if (pl.nv == 4 && pl.tile == 16) return LAUNCH<TE, 4, 16, TMA>(__VA_ARGS__);    \
    return SBDA_ERR_UNSUPPORTED;                                                    \
  } while (0)

template <typename TE, bool TMA>
int fwd_tiles(const FwdMaps& maps, const FwdParams& p, const Plan& pl, cudaStream_t st) {
  SBDA_FOR_TILES(launch_fwd, TE, TMA, maps, p, pl, st);
}
template <typename TE, bool TMA>
int bwd_tiles(const BwdMaps& maps, const BwdParams& p, const Plan& pl, cudaStream_t st) {
  SBDA_FOR_TILES(launch_bwd, TE, TMA, maps, p, pl, st);
}

template <bool TMA>
int fwd_dtype(int dtype, const FwdMaps& maps, const FwdParams& p, const Plan& pl, cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return fwd_tiles<float, TMA>(maps, p, pl, st);
  if (dtype == SBDA_DTYPE_F16) return fwd_tiles<__half, TMA>(maps, p, pl, st);
  return fwd_tiles<__nv_bfloat16, TMA>(maps, p, pl, st);
}
template <bool TMA>
int bwd_dtype(int dtype, const BwdMaps& maps, const BwdParams& p, const Plan& pl, cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return bwd_tiles<float, TMA>(maps, p, pl, st);
  if (dtype == SBDA_DTYPE_F16) return bwd_tiles<__half, TMA>(maps, p, pl, st);
  return bwd_tiles<__nv_bfloat16, TMA>(maps, p, pl, st);
}

}  // namespace sbda

using namespace sbda;

extern "C" int sbda_b200_abi_version(void) { return SBDA_B200_ABI_VERSION; }

extern "C" const char* sbda_b200_status_string(int status) {
  switch (status) {
    case SBDA_OK: return "ok";
    case SBDA_ERR_INVALID: return "invalid argument (shape, stride, offsets or pointer)";
    case SBDA_ERR_DTYPE: return "unsupported SBDA dtype";
    case SBDA_ERR_UNSUPPORTED: return "offsets or shape outside the kernel envelope";
    case SBDA_ERR_CUDA: return "CUDA runtime error";
    case SBDA_ERR_DEVICE: return "device-side fault reported by an SBDA kernel";
    default: return "unknown SBDA status";
  }
}

extern "C" int sbda_b200_forward(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                 float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v, sbda_tensor out,
                                 float* lse, void* stream) {
  int st = validate(dtype, shape, offsets, n_offsets);
  if (st != SBDA_OK) return st;
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, L = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || L == 0) return SBDA_OK;
  if (!q.data || !k.data || !v.data || !out.data || !lse) return SBDA_ERR_INVALID;
  const int e = elem_size(dtype);
  Plan pl;
  st = make_plan(offsets, n_offsets, L, D, e, &pl);
  if (st != SBDA_OK) return st;

  FwdParams p;
  memset(&p, 0, sizeof(p));
  p.B = (int)B;
  p.H = (int)H;
  p.Hkv = (int)Hkv;
  p.G = (int)(H / Hkv);
  p.L = (int)L;
  p.D = (int)D;
  p.scale = scale;
  p.g = pl.g;
  p.q = arg_of(q);
  p.k = arg_of(k);
  p.v = arg_of(v);
  p.out = arg_of(out);
  p.lse = lse;

  FwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  bool tma = vector_ok(q, B, H, L, D, e) && vector_ok(k, B, Hkv, L, D, e) && vector_ok(v, B, Hkv, L, D, e) &&
             vector_ok(out, B, H, L, D, e);
  if (tma) {
    unsigned dummy;
    tma = encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.kT, &p.slots_k, k, dtype, B, Hkv, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.vT, &p.slots_v, v, dtype, B, Hkv, L, D, pl.pitch, pl.tile);
    if (tma && pl.g.Hn > 0)
      tma = encode_map(&maps.kH, &dummy, k, dtype, B, Hkv, L, D, pl.pitch, pl.g.Hn) &&
            encode_map(&maps.vH, &dummy, v, dtype, B, Hkv, L, D, pl.pitch, pl.g.Hn);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return tma ? fwd_dtype<true>(dtype, maps, p, pl, s) : fwd_dtype<false>(dtype, maps, p, pl, s);
}

extern "C" int sbda_b200_backward(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                  float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                                  sbda_tensor grad_out, const float* lse, sbda_tensor grad_q,
                                  sbda_tensor grad_k, sbda_tensor grad_v, void* stream) {
  int st = validate(dtype, shape, offsets, n_offsets);
  if (st != SBDA_OK) return st;
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, L = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || L == 0) return SBDA_OK;
  if (!q.data || !k.data || !v.data || !grad_out.data || !lse || !grad_q.data || !grad_k.data ||
      !grad_v.data)
    return SBDA_ERR_INVALID;
  const int e = elem_size(dtype);
  Plan pl;
  st = make_plan(offsets, n_offsets, L, D, e, &pl);
  if (st != SBDA_OK) return st;

  BwdParams p;
  memset(&p, 0, sizeof(p));
  p.B = (int)B;
  p.H = (int)H;
  p.Hkv = (int)Hkv;
  p.G = (int)(H / Hkv);
  p.L = (int)L;
  p.D = (int)D;
  p.scale = scale;
  p.g = pl.g;
  p.q = arg_of(q);
  p.k = arg_of(k);
  p.v = arg_of(v);
  p.dout = arg_of(grad_out);
  p.dq = arg_of(grad_q);
  p.dk = arg_of(grad_k);
  p.dv = arg_of(grad_v);
  p.lse = lse;

  BwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  bool tma = vector_ok(q, B, H, L, D, e) && vector_ok(k, B, Hkv, L, D, e) && vector_ok(v, B, Hkv, L, D, e) &&
             vector_ok(grad_out, B, H, L, D, e) && vector_ok(grad_q, B, H, L, D, e) &&
             vector_ok(grad_k, B, Hkv, L, D, e) && vector_ok(grad_v, B, Hkv, L, D, e);
  if (tma) {
    unsigned dummy;
    tma = encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.dT, &p.slots_d, grad_out, dtype, B, H, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.kT, &p.slots_k, k, dtype, B, Hkv, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.vT, &p.slots_v, v, dtype, B, Hkv, L, D, pl.pitch, pl.tile);
    if (tma && pl.g.Hn > 0)
      tma = encode_map(&maps.qH, &dummy, q, dtype, B, H, L, D, pl.pitch, pl.g.Hn) &&
            encode_map(&maps.dH, &dummy, grad_out, dtype, B, H, L, D, pl.pitch, pl.g.Hn) &&
            encode_map(&maps.kH, &dummy, k, dtype, B, Hkv, L, D, pl.pitch, pl.g.Hn) &&
            encode_map(&maps.vH, &dummy, v, dtype, B, Hkv, L, D, pl.pitch, pl.g.Hn);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return tma ? bwd_dtype<true>(dtype, maps, p, pl, s) : bwd_dtype<false>(dtype, maps, p, pl, s);
}

extern "C" int sbda_b200_device_status(uint32_t* flags_out, int reset) {
  unsigned value = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return SBDA_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&value, g_device_status, sizeof(value)) != cudaSuccess) return SBDA_ERR_CUDA;
  if (reset) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero)) != cudaSuccess) return SBDA_ERR_CUDA;
  }
  if (flags_out) *flags_out = value;
  return value ? SBDA_ERR_DEVICE : SBDA_OK;
}
