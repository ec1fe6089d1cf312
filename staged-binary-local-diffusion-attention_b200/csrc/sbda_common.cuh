// sbda_common.cuh -- shared device helpers and launch structures of the SBDA
// sm_100a kernels (mbarrier / TMA inline PTX, element packing, row staging).
#pragma once

#include "sbda_b200.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <math.h>
#include <stdint.h>

namespace sbda {

constexpr int kThreads = 128;             // 4 warps
constexpr int kGroups = kThreads / 8;     // 8-lane row groups per CTA
constexpr unsigned kFaultWaitExpired = 1u;

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

// Contiguous sequence shards: rank r holds positions [r * shard_len,
// (r + 1) * shard_len) of a sequence of total_len positions.  One GPU is the
// case world = 1, shard_len = total_len, pos0 = 0.
constexpr int kMaxShards = 8;
struct ShardInfo {
  int rank, world;
  int shard_len;                 // positions per rank
  int pos0;                      // global position of local row 0
  int total_len;                 // positions of the whole sequence
  const float* lse[kMaxShards];  // per-rank log-sum-exp bases [B, H, shard_len] (backward)
};

struct FwdParams {
  int B, H, Hkv, G, L, D;
  float scale;
  Geometry g;
  TensorArg q, k, v, out;
  float* lse;
  unsigned slots_q, slots_k, slots_v;
  unsigned* status;
  ShardInfo sh;
};

struct BwdParams {
  int B, H, Hkv, G, L, D;
  float scale;
  Geometry g;
  TensorArg q, k, v, dout, dq, dk, dv;
  const float* lse;
  unsigned slots_q, slots_k, slots_v, slots_d;
  unsigned* status;
  ShardInfo sh;
};

// Tensor maps: *T = TILE-row box, *H = Hn-row halo box.
struct FwdMaps {
  CUtensorMap qT, kT, vT, kH, vH;
};
struct BwdMaps {
  CUtensorMap qT, qH, dT, dH, kT, kH, vT, vH;
  CUtensorMap lseT;  // windowed backward: fp32 [B*H, L] rows, box of the Q/dO slot height (rounded to 32)
};

// Sequence-sharded maps: one map per rank over that rank's buffer (peer
// memory mapped into this process), selected per staged region by its owner.
struct ShardFwdMaps {
  CUtensorMap qT, kT[kMaxShards], kH[kMaxShards], vT[kMaxShards], vH[kMaxShards];
};
struct ShardBwdMaps {
  CUtensorMap qT[kMaxShards], qH[kMaxShards], dT[kMaxShards], dH[kMaxShards];
  CUtensorMap kT[kMaxShards], kH[kMaxShards], vT[kMaxShards], vH[kMaxShards];
  // LSE rows (fp32 [B*H, L] per rank): lseT boxes one tile, lseH the halo rows
  // past it (rounded up to 4), each from the rank that owns them.
  CUtensorMap lseT[kMaxShards], lseH[kMaxShards];
};

// Map and map coordinate of the rows starting at global position gpos.
// One GPU: the map itself.  Shards: the owning rank's map; positions outside
// the sequence use this rank's map at an out-of-range coordinate, which the
// copy engine zero-fills.
__device__ __forceinline__ const CUtensorMap* pick_map(const CUtensorMap& m, const ShardInfo& s, int gpos,
                                                       int& coord) {
  coord = gpos - s.pos0;
  return &m;
}
__device__ __forceinline__ const CUtensorMap* pick_map(const CUtensorMap (&m)[kMaxShards], const ShardInfo& s,
                                                       int gpos, int& coord) {
  // Most boxes are this rank's rows: one compare.  Otherwise the owner is the
  // number of shard starts at or below gpos (no integer division on the path
  // that issues the copies).
  int owner = s.rank;
  if ((unsigned)(gpos - s.pos0) >= (unsigned)s.shard_len && gpos >= 0 && gpos < s.total_len) {
    owner = 0;
#pragma unroll
    for (int r = 1; r < kMaxShards; ++r) owner += gpos >= (long long)r * s.shard_len ? 1 : 0;
  }
  coord = gpos - owner * s.shard_len;
  return &m[owner];
}

// This rank's own map (one GPU: the map itself), and whether the call's local
// rows [lo, hi) all lie in this rank's shard, so that every box over them can use
// that map at local coordinates without an owner search.  One GPU: always (rows
// outside the sequence read as the map's zero fill).  The copies of a step are
// issued by one thread on the step's critical path; the owner search for each of
// a step's boxes was most of the sharded kernels' extra time.
__device__ __forceinline__ const CUtensorMap* own_map(const CUtensorMap& m, const ShardInfo&) { return &m; }
__device__ __forceinline__ const CUtensorMap* own_map(const CUtensorMap (&m)[kMaxShards], const ShardInfo& s) {
  return &m[s.rank];
}
__device__ __forceinline__ bool own_rows(const CUtensorMap&, const ShardInfo&, int, int) { return true; }
__device__ __forceinline__ bool own_rows(const CUtensorMap (&)[kMaxShards], const ShardInfo& s, int lo, int hi) {
  return lo >= 0 && hi <= s.shard_len;
}

// Log-sum-exp of (b, h) at global position q (0 <= q < total_len).
__device__ __forceinline__ float lse_at(const ShardInfo& s, long long bh, int q) {
  const int owner = s.world == 1 ? 0 : q / s.shard_len;
  return s.lse[owner][bh * s.shard_len + (q - owner * s.shard_len)];
}

// --------------------------------------------------------------------------
// Programmatic dependent launch.  The windowed kernels are launched with
// programmatic stream serialization (launch_chained): their CTAs may be
// scheduled while the previous kernel on the stream drains its last wave, and
// they call grid_dependency_sync() before their first global memory access,
// which waits until that kernel has completed and its writes are visible.  The
// same call lets the next chained kernel be scheduled once every CTA of this
// grid has started.  Without the launch attribute both instructions are no-ops.
// --------------------------------------------------------------------------

__device__ __forceinline__ void grid_dependency_sync() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... Params, typename... Args>
inline cudaError_t launch_chained(void (*kern)(Params...), unsigned grid, size_t smem, cudaStream_t st,
                                  const Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr = {};
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

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
__device__ __forceinline__ void fault_and_drain(unsigned* status, uint64_t* bar, uint32_t parity) {
  if (threadIdx.x == 0 && status) atomicOr(status, kFaultWaitExpired);
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

// 2-D tiled TMA load (fp32 LSE rows): coordinate 0 = position (a multiple of
// 4, so the 16-byte rule on the innermost coordinate holds), 1 = batch*head.
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1)
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
// Packed fp32 pairs (sm_100 f32x2 ALU ops): one instruction per two lanes of
// math, used for the dot products and the axpy updates of every row.
// --------------------------------------------------------------------------

__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 2^x on the special-function unit (ex2.approx: relative error ~2^-22).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Eight consecutive channels of one row held by one lane, as four pairs.
struct Frag {
  float2 v[4];
};

__device__ __forceinline__ Frag frag_zero() {
  Frag f;
#pragma unroll
  for (int i = 0; i < 4; ++i) f.v[i] = make_float2(0.f, 0.f);
  return f;
}

template <typename TE>
struct FragIO;

// 16-bit rows: a lane owns one 16-byte vector (8 elements) at byte l*16.
template <>
struct FragIO<__nv_bfloat16> {
  static constexpr int kLaneBytes = 16;
  static __device__ __forceinline__ Frag load(const uint8_t* row, int l) {
    return from_words(reinterpret_cast<const uint4*>(row + l * 16));
  }
  static __device__ __forceinline__ Frag from_words(const uint4* w) {
    const uint4 u = w[0];
    Frag f;
    f.v[0] = make_float2(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u));
    f.v[1] = make_float2(__uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
    f.v[2] = make_float2(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xffff0000u));
    f.v[3] = make_float2(__uint_as_float(u.w << 16), __uint_as_float(u.w & 0xffff0000u));
    return f;
  }
  static __device__ __forceinline__ uint4 pack(const Frag& f) {
    return make_uint4(Elem<__nv_bfloat16>::pack2(f.v[0].x, f.v[0].y), Elem<__nv_bfloat16>::pack2(f.v[1].x, f.v[1].y),
                      Elem<__nv_bfloat16>::pack2(f.v[2].x, f.v[2].y), Elem<__nv_bfloat16>::pack2(f.v[3].x, f.v[3].y));
  }
};

template <>
struct FragIO<__half> {
  static constexpr int kLaneBytes = 16;
  static __device__ __forceinline__ Frag load(const uint8_t* row, int l) {
    return from_words(reinterpret_cast<const uint4*>(row + l * 16));
  }
  static __device__ __forceinline__ Frag from_words(const uint4* w) {
    const uint4 u = w[0];
    Frag f;
    f.v[0] = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    f.v[1] = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    f.v[2] = __half22float2(*reinterpret_cast<const __half2*>(&u.z));
    f.v[3] = __half22float2(*reinterpret_cast<const __half2*>(&u.w));
    return f;
  }
  static __device__ __forceinline__ uint4 pack(const Frag& f) {
    return make_uint4(Elem<__half>::pack2(f.v[0].x, f.v[0].y), Elem<__half>::pack2(f.v[1].x, f.v[1].y),
                      Elem<__half>::pack2(f.v[2].x, f.v[2].y), Elem<__half>::pack2(f.v[3].x, f.v[3].y));
  }
};

// fp32 rows: a lane owns two 16-byte vectors (8 elements) at byte l*32.
template <>
struct FragIO<float> {
  static constexpr int kLaneBytes = 32;
  static __device__ __forceinline__ Frag load(const uint8_t* row, int l) {
    return from_words(reinterpret_cast<const uint4*>(row + l * 32));
  }
  static __device__ __forceinline__ Frag from_words(const uint4* w) {
    const float4 a = *reinterpret_cast<const float4*>(&w[0]);
    const float4 b = *reinterpret_cast<const float4*>(&w[1]);
    Frag f;
    f.v[0] = make_float2(a.x, a.y);
    f.v[1] = make_float2(a.z, a.w);
    f.v[2] = make_float2(b.x, b.y);
    f.v[3] = make_float2(b.z, b.w);
    return f;
  }
};

// One lane's part of a row read straight from global memory, still packed
// (16-byte words).  Vector layouts only: 16-byte aligned rows, unit channel
// stride, D * element size a multiple of 16.  Channels past D, and every
// channel when `live` is false, read as zero.
template <typename TE>
struct RowWords {
  uint4 w[FragIO<TE>::kLaneBytes / 16];
};

template <typename TE>
__device__ __forceinline__ RowWords<TE> load_row_words(const TE* row, int D, int l, bool live) {
  constexpr int kEpw = 16 / sizeof(TE);  // elements per 16-byte word
  RowWords<TE> r;
#pragma unroll
  for (int i = 0; i < FragIO<TE>::kLaneBytes / 16; ++i) {
    const int c = l * 8 + i * kEpw;
    r.w[i] = make_uint4(0u, 0u, 0u, 0u);
    if (live && c < D) r.w[i] = __ldg(reinterpret_cast<const uint4*>(row + c));
  }
  return r;
}

__device__ __forceinline__ float frag_dot(const Frag& a, const Frag& b) {
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 4; ++i) acc = fma2(a.v[i], b.v[i], acc);
  return acc.x + acc.y;
}

// acc += w * x
__device__ __forceinline__ void frag_axpy(Frag& acc, float w, const Frag& x) {
  const float2 ww = make_float2(w, w);
#pragma unroll
  for (int i = 0; i < 4; ++i) acc.v[i] = fma2(ww, x.v[i], acc.v[i]);
}

__device__ __forceinline__ void frag_scale(Frag& acc, float w) {
  const float2 ww = make_float2(w, w);
#pragma unroll
  for (int i = 0; i < 4; ++i) acc.v[i] = mul2(ww, acc.v[i]);
}

// acc = w * x
__device__ __forceinline__ Frag frag_mul(float w, const Frag& x) {
  const float2 ww = make_float2(w, w);
  Frag r;
#pragma unroll
  for (int i = 0; i < 4; ++i) r.v[i] = mul2(ww, x.v[i]);
  return r;
}

__device__ __forceinline__ void frag_add(Frag& acc, const Frag& x) {
#pragma unroll
  for (int i = 0; i < 4; ++i) acc.v[i] = add2(acc.v[i], x.v[i]);
}

// Stores a lane's 8 channels of a row (channels [8l, 8l+8) of D).
template <typename TE, bool VEC>
__device__ __forceinline__ void store_frag(TE* row, long long sd, int D, int l, const Frag& f) {
  const int c0 = l * 8;
  if (c0 >= D) return;
  if constexpr (VEC) {
    if constexpr (sizeof(TE) == 2) {
      *reinterpret_cast<uint4*>(row + c0) = FragIO<TE>::pack(f);
    } else {
      *reinterpret_cast<float4*>(row + c0) = make_float4(f.v[0].x, f.v[0].y, f.v[1].x, f.v[1].y);
      if (c0 + 4 < D)
        *reinterpret_cast<float4*>(row + c0 + 4) = make_float4(f.v[2].x, f.v[2].y, f.v[3].x, f.v[3].y);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (c0 + 2 * i < D) row[(long long)(c0 + 2 * i) * sd] = Elem<TE>::from_float(f.v[i].x);
      if (c0 + 2 * i + 1 < D) row[(long long)(c0 + 2 * i + 1) * sd] = Elem<TE>::from_float(f.v[i].y);
    }
  }
}

// Sum over the LPR lanes of a row group (xor butterfly within the group).
template <int LPR>
__device__ __forceinline__ float lane_group_sum(float x) {
#pragma unroll
  for (int m = LPR / 2; m >= 1; m >>= 1) x += __shfl_xor_sync(0xffffffffu, x, m);
  return x;
}

// Reduce-scatter over the 8 lanes of a row group of four (x[s], x[s + 4]) pairs
// (lane index l = lane % 8): the group totals of x[l & 3] and x[(l & 3) + 4]
// out on lanes l and l ^ 4: two halving exchanges (4 + 2 shuffles), then an
// exchange of both values between lanes l and l ^ 4 (2 shuffles).  Both lanes of
// a source then hold its q.k and dO.v, so its softmax terms need no further
// exchange before the sum over sources.
__device__ __forceinline__ float2 group8_reduce_scatter_pairs(const float (&x)[8], int l) {
  const unsigned full = 0xffffffffu;
  const bool h1 = l & 1, h2 = l & 2;
  float w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float send = h1 ? x[2 * j] : x[2 * j + 1];
    w[j] = (h1 ? x[2 * j + 1] : x[2 * j]) + __shfl_xor_sync(full, send, 1);
  }
  float z[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float send = h2 ? w[2 * j] : w[2 * j + 1];
    z[j] = (h2 ? w[2 * j + 1] : w[2 * j]) + __shfl_xor_sync(full, send, 2);
  }
  return make_float2(z[0] + __shfl_xor_sync(full, z[0], 4), z[1] + __shfl_xor_sync(full, z[1], 4));
}

// Four per-lane partial sums over the 8 lanes of a row group: the group total
// of x[k] out on lanes 2k and 2k + 1.
__device__ __forceinline__ float group8_reduce_scatter4(const float (&x)[4], int l) {
  const unsigned full = 0xffffffffu;
  const bool h4 = l & 4, h2 = l & 2;
  float w[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = h4 ? x[i] : x[i + 2];
    w[i] = (h4 ? x[i + 2] : x[i]) + __shfl_xor_sync(full, send, 4);
  }
  const float send = h2 ? w[0] : w[1];
  const float z = (h2 ? w[1] : w[0]) + __shfl_xor_sync(full, send, 2);
  return z + __shfl_xor_sync(full, z, 1);
}

// --------------------------------------------------------------------------
// v2 launch structures (windowed / chain-walking kernels, MHA)
// --------------------------------------------------------------------------

struct V2Geometry {
  int has0, has1, has2;  // near sources (offsets 0, 1, 2) present
  int has_far, d;        // far source: offset d > 2
  int nT;                // tiles per (batch, head)
  int R, A, rem;         // chain order of tiles (forward launch order)
  int mode;              // backward: 0 = chain walk (d % TILE == 0, d >= TILE), 1 = local tiles,
                         // 2 = local carry (far d < TILE, d % 4 == 0)
  int halo;              // backward: consumer halo rows past the tile (2, or d in mode 1)
  int seg;               // backward: tiles per CTA
  int segs;              // backward: segments per chain (mode 0) or per (b, h) (mode 1)
  int chains;            // backward chain walks per (b, h): min(R, nT)
};

// Per-head RMSNorm + RoPE of q or k applied inside the windowed kernels (the
// *_normed entry points): fp32 weight [D], the cos/sin table [rows, D / 2] in
// the element type, and the table row of local position 0.
struct NormRopeArgs {
  const float* w;
  const void* cos_t;
  const void* sin_t;
  long long table_offset;
  float eps;
};

struct FwdV2Params {
  int B, H, L, D;        // L: positions of this call's rows (the shard when sharded)
  int G;                 // query heads per kv head (1 = MHA); K/V rows come from kv head h / G
  float scale;
  V2Geometry g;
  TensorArg q, k, v, out;
  float* lse;
  unsigned slots_q, slots_k, slots_v;
  unsigned* status;
  ShardInfo sh;          // one shard (pos0 = 0, total_len = L) unless sequence-sharded
  NormRopeArgs nq, nk;   // normed kernels only: q and k arrive raw
};

struct BwdV2Params {
  int B, H, L, D;        // L: positions of this call's rows (the shard when sharded)
  int G;                 // query heads per kv head (1 = MHA); K/V rows come from kv head h / G
  float scale;
  V2Geometry g;
  TensorArg q, k, v, dout, dq, dk, dv;
  const float* lse;
  unsigned slots_q, slots_k, slots_v, slots_d;
  unsigned* status;
  int lse_tma;   // 1: LSE rows staged by the copy engine with Q/dO (L % 4 == 0)
  int lse_box;   // rows of an LSE slot in shared memory (Q/dO slot height rounded up to 32)
  int lse_tx;    // bytes the LSE copies of one step deliver
  ShardInfo sh;  // one shard (pos0 = 0, total_len = L) unless sequence-sharded
  NormRopeArgs nq, nk;  // normed kernels only: q and k arrive raw, dq and dk leave raw
  float* dw_partial;    // normed kernels only: [gridDim.x, 2, 64] per-CTA norm-weight gradients (q, k)
};

// Uniform kernels (sbda_v3.cu): every source a shifted tile.
struct V3Params {
  int B, H, Hkv, G, L, D;
  float scale;
  int S;
  int off[4];
  int nT;
  int o_min, s_q;  // smallest offset and its source index (the dQ writer)
  TensorArg q, k, v, out, dout, dq, dk, dv;
  float* lse;      // forward writes, backward reads
  const uint8_t* mask;  // optional [B, L]: bit s of row i allows source s (null = all)
  unsigned slots_q, slots_k, slots_v, slots_d;
  unsigned* status;
};

struct V3Plan {
  int lpr, tile, pitch;
  size_t smem_fwd, smem_bwd;
};

// v2 tile height for a row pitch: each of the 128/LPR row groups owns a run of
// four consecutive rows.
__host__ __device__ constexpr int v2_tile(int lpr) { return 4 * (kThreads / lpr); }

// Floats of the backward's softmax-record ring for tile height T: 2T records of
// 8 floats plus 4 floats of padding per 4 records.
__host__ __device__ constexpr int v2_ring_floats(int T) { return 2 * T * 8 + (2 * T / 4) * 4; }

// Host helpers shared by the translation units (sbda_api.cu): the device's
// fault word (kernels report expired waits into it) and its SM count.
unsigned* status_ptr();
int sm_count();

// Untiled bulk copy global -> this CTA's shared memory, completion counted on
// `bar` (both addresses 16-byte aligned, `bytes` a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// Host-side launchers (defined in sbda_v1.cu / sbda_v2.cu).
struct Plan {
  int tile;
  int nv;
  int pitch;
  Geometry g;
  size_t smem_fwd, smem_bwd;
};

int v1_forward(int dtype, bool tma, const FwdMaps& maps, const FwdParams& p, const Plan& pl, cudaStream_t st);
int v1_backward(int dtype, bool tma, const BwdMaps& maps, const BwdParams& p, const Plan& pl, cudaStream_t st);
int v1_forward_sharded(int dtype, const ShardFwdMaps& maps, const FwdParams& p, const Plan& pl, cudaStream_t st);
int v1_backward_sharded(int dtype, const ShardBwdMaps& maps, const BwdParams& p, const Plan& pl, cudaStream_t st);

struct V2Plan {
  int lpr;
  int tile;
  int pitch;
  int lse_box;
  V2Geometry g;
  size_t smem_fwd, smem_bwd;
  unsigned blocks_bwd;
};

int v2_forward(int dtype, bool tma, const FwdMaps& maps, const FwdV2Params& p, const V2Plan& pl, cudaStream_t st);
int v2_forward_sharded(int dtype, const ShardFwdMaps& maps, const FwdV2Params& p, const V2Plan& pl,
                       cudaStream_t st);
int v2_backward_sharded(int dtype, const ShardBwdMaps& maps, const BwdV2Params& p, const V2Plan& pl,
                        cudaStream_t st);
int v3_forward(int dtype, bool tma, const FwdMaps& maps, const V3Params& p, const V3Plan& pl, cudaStream_t st);
int v3_backward(int dtype, bool tma, const BwdMaps& maps, const V3Params& p, const V3Plan& pl, cudaStream_t st);
int v2_backward(int dtype, bool tma, const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl,
                cudaStream_t st);

// Windowed kernels with the per-head RMSNorm + RoPE fused in (sbda_v2_normed.cu).
bool v2_normed_plan_ok(const V2Plan& pl);
int v2_forward_normed(int dtype, const FwdMaps& maps, const FwdV2Params& p, const V2Plan& pl, cudaStream_t st);
int64_t v2_normed_workspace_floats(unsigned blocks);

// Grouped-query attention on the windowed backward (sbda_v2_grouped.cu): fp32
// per-query-head dK/dV partials in `workspace`, then a fixed-order group sum.
bool v2_grouped_plan_ok(const V2Plan& pl);
int v2_backward_grouped(int dtype, const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl, const float* workspace,
                        int Hkv, const TensorArg& dk, const TensorArg& dv, cudaStream_t st);
int v2_backward_normed(int dtype, const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl, float* grad_q_w,
                       float* grad_k_w, float* workspace, cudaStream_t st);

}  // namespace sbda
