// sbda_v2_kernels.cuh -- windowed SBDA kernels for the MHA schedules of the SBDA
// family: near offsets within {0, 1, 2} plus at most one far offset d > 2.
//
// Same function as the reference's fused op (BiAttn/sbda_triton.py:1290-1360:
// forward O and softmax statistics, key-centric gather backward) and its eager
// oracle (BiAttn/left_v2.py:335-405).
//
// What differs from the general kernels (sbda_v1.cu):
//  * A row group of LPR lanes owns a run of four consecutive rows, so the K/V
//    rows of offsets 1 and 2 are the rows of offsets 0 of the previous two
//    iterations: they stay unpacked in registers (a sliding window) instead of
//    being re-read and re-converted, and every multiply-add runs on packed
//    fp32 pairs (fma.rn.f32x2).
//  * The backward walks dyadic chains.  When d is a multiple of the tile
//    height, a CTA processes tiles t, t-R, t-2R, ... (R = d / TILE) of one
//    (batch, head): the far edge of consumer j0+r feeds key j0+r-d, which is
//    row r of the next tile of the walk, so its dK/dV contribution is carried
//    in the same lanes' registers to the next step.  No consumer is computed
//    twice except one "pre" tile per CTA segment, and the K/V tile staged as
//    this step's far sources is the next step's near sources.  Two K/V slots
//    alternate: phase 2 (the key gather) reads no K/V, so the next step's far
//    tile is fetched into this step's near slot as soon as phase 1 is done;
//    Q/dO are double-buffered and fetched a whole step ahead.
//  * For d < TILE with d % 4 == 0 whose local staging (below) would keep fewer
//    than three CTAs on an SM ("local carry" mode) a CTA walks consecutive
//    tiles downwards.  In the key gather, row group g takes keys
//    4g - d .. 4g - d + 3 (mod TILE), so the far consumer of each of its keys
//    is one of its own rows 4g .. 4g + 3: in this tile, or (for the last d
//    keys) in the tile of the step before, whose contribution the same lanes
//    carried in registers.  No consumer is computed twice except one carry-only
//    "pre" tile per CTA segment.
//  * Other d < TILE ("local" mode): the keys of a tile also need the d
//    consumers past its end, recomputed by the first step of a walk; later
//    steps take them from the step before (next point).
//  * The softmax records of a step live in a ring of two tiles: in a walk of
//    consecutive tiles the consumers past this tile's end are the first rows
//    of the previous step's tile, so only the first step computes them.
//  * Sequence shards: a call covers one rank's rows; every TMA box lies in one
//    rank's shard (tiles, in-tile halos, d-aligned chain tiles), so the box's
//    map is the owner's (pick_map).  Masks use global positions, LSE rows past
//    the shard are read from their owner, and a walk's pre tile may be the next
//    rank's.  One shard (pos0 = 0, total_len = L) is the unsharded case.

#pragma once

#include <type_traits>

#include "sbda_common.cuh"

namespace sbda {

__device__ __forceinline__ int chain_tile_v2(int idx, int R, int A, int rem) {
  if (R == 0) return idx;
  const int full = rem * A;
  int r, a;
  if (idx < full) {
    r = idx / A;
    a = idx - r * A;
  } else {
    const int j = idx - full, a1 = A - 1;
    r = rem + j / a1;
    a = j - (j / a1) * a1;
  }
  return a * R + r;
}

// --------------------------------------------------------------------------
// Per-head RMSNorm + half-split RoPE inside the kernels (head_dim 64, 8 lanes
// per row: lane l holds channels 8l .. 8l + 7, so the rotation partner of
// channel j, j -+ 32, is in lane l ^ 4).  Reference arithmetic
// (BiAttn/attention_common.py:13-22, 44-49, 72-76):
//   r = rsqrt(mean(x^2) + eps) in fp32,  y = cast(x * r * w),
//   z_j      = cast(cast(y_j c_j) - cast(y_{j+32} s_j)),
//   z_{j+32} = cast(cast(y_{j+32} c_j) + cast(y_j s_j)),
// with (c, s) the position's table row (fp32 angles cast to the element type).
// 16-bit types run the RoPE on packed pairs (one rounding per op, like the
// reference's eager ops); fp32 rounds each op to fp32.
// --------------------------------------------------------------------------

template <typename TE>
struct PackedOps;
template <>
struct PackedOps<__nv_bfloat16> {
  using P2 = __nv_bfloat162;
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    const P2 r = __hmul2(*reinterpret_cast<const P2*>(&a), *reinterpret_cast<const P2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    const P2 r = __hadd2(*reinterpret_cast<const P2*>(&a), *reinterpret_cast<const P2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    const P2 r = __hsub2(*reinterpret_cast<const P2*>(&a), *reinterpret_cast<const P2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
};
template <>
struct PackedOps<__half> {
  using P2 = __half2;
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    const P2 r = __hmul2(*reinterpret_cast<const P2*>(&a), *reinterpret_cast<const P2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    const P2 r = __hadd2(*reinterpret_cast<const P2*>(&a), *reinterpret_cast<const P2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    const P2 r = __hsub2(*reinterpret_cast<const P2*>(&a), *reinterpret_cast<const P2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
};

// 1 / sqrt(x) on the special-function unit.  Its arguments here are
// mean(x^2) + eps >= eps > 0, never denormal, so the flush-to-zero form gives
// what rsqrtf gives without rsqrtf's denormal handling.
__device__ __forceinline__ float nr_rsqrt(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The lane's 8 weights (fp32).
__device__ __forceinline__ Frag nr_weights(const float* w, int l) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(w + 8 * l));
  const float4 b = __ldg(reinterpret_cast<const float4*>(w + 8 * l + 4));
  Frag f;
  f.v[0] = make_float2(a.x, a.y);
  f.v[1] = make_float2(a.z, a.w);
  f.v[2] = make_float2(b.x, b.y);
  f.v[3] = make_float2(b.z, b.w);
  return f;
}

// Sum over the row's 8 lanes of sum_k a_k b_k (this lane's channels).
__device__ __forceinline__ float nr_row_dot(const Frag& a, const Frag& b) {
  float2 acc = mul2(a.v[0], b.v[0]);
#pragma unroll
  for (int i = 1; i < 4; ++i) acc = fma2(a.v[i], b.v[i], acc);
  return group_sum(acc.x + acc.y);
}

// Table row of position pos (clamped into the sequence: rows outside it are
// zero and stay zero whatever the table says).
template <typename TE>
__device__ __forceinline__ const TE* nr_table_row(const void* table, const NormRopeArgs& a, int pos, int L) {
  const int p = pos < 0 ? 0 : (pos >= L ? L - 1 : pos);
  return reinterpret_cast<const TE*>(table) + (a.table_offset + p) * 32;
}

// The lane's cos and sin table words of one position (its 8 entries of each:
// channels 8 (l & 3) .. 8 (l & 3) + 7 of the half-width table row).  Loading
// them apart from their use lets callers issue the loads early: the table is
// too large to stay in L1, and a load issued just before its use puts a round
// trip to L2 on the row's dependency chain.
template <typename TE>
struct RopeWords {
  uint4 c[FragIO<TE>::kLaneBytes / 16], s[FragIO<TE>::kLaneBytes / 16];
};

template <typename TE>
__device__ __forceinline__ RopeWords<TE> rope_words(const NormRopeArgs& a, int pos, int L, int l) {
  const uint4* ct = reinterpret_cast<const uint4*>(nr_table_row<TE>(a.cos_t, a, pos, L) + 8 * (l & 3));
  const uint4* st = reinterpret_cast<const uint4*>(nr_table_row<TE>(a.sin_t, a, pos, L) + 8 * (l & 3));
  RopeWords<TE> rw;
#pragma unroll
  for (int i = 0; i < FragIO<TE>::kLaneBytes / 16; ++i) {
    rw.c[i] = __ldg(ct + i);
    rw.s[i] = __ldg(st + i);
  }
  return rw;
}

// Normalised and rotated channels of one lane (fp32 values of the element-type
// results) from the position's table words; r_out receives the row's rsqrt
// (the backward's Jacobian needs it).
template <typename TE>
__device__ __forceinline__ Frag norm_rope_frag_w(const Frag& x, int l, const Frag& w, float eps,
                                                 const RopeWords<TE>& rw, float* r_out) {
  const unsigned full = 0xffffffffu;
  const float r = nr_rsqrt(fmaf(nr_row_dot(x, x), 1.f / 64.f, eps));
  if (r_out) *r_out = r;
  const float2 rr = make_float2(r, r);
  if constexpr (sizeof(TE) == 2) {
    using Ops = PackedOps<TE>;
    uint32_t y[4], z[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 n = mul2(x.v[i], rr);
      const float2 yw = mul2(n, w.v[i]);
      y[i] = Elem<TE>::pack2(yw.x, yw.y);
    }
    const uint4 cw = rw.c[0], sw = rw.s[0];
    const uint32_t c[4] = {cw.x, cw.y, cw.z, cw.w}, s[4] = {sw.x, sw.y, sw.z, sw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t partner = __shfl_xor_sync(full, y[i], 4);
      const uint32_t t1 = Ops::mul(y[i], c[i]), t2 = Ops::mul(partner, s[i]);
      z[i] = l < 4 ? Ops::sub(t1, t2) : Ops::add(t1, t2);
    }
    const uint4 zw = make_uint4(z[0], z[1], z[2], z[3]);
    return FragIO<TE>::from_words(&zw);
  } else {
    const float4 c0 = *reinterpret_cast<const float4*>(&rw.c[0]), c1 = *reinterpret_cast<const float4*>(&rw.c[1]);
    const float4 s0 = *reinterpret_cast<const float4*>(&rw.s[0]), s1 = *reinterpret_cast<const float4*>(&rw.s[1]);
    const float2 c[4] = {make_float2(c0.x, c0.y), make_float2(c0.z, c0.w), make_float2(c1.x, c1.y),
                         make_float2(c1.z, c1.w)};
    const float2 s[4] = {make_float2(s0.x, s0.y), make_float2(s0.z, s0.w), make_float2(s1.x, s1.y),
                         make_float2(s1.z, s1.w)};
    Frag z;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 y = mul2(mul2(x.v[i], rr), w.v[i]);
      const float2 partner = make_float2(__shfl_xor_sync(full, y.x, 4), __shfl_xor_sync(full, y.y, 4));
      const float2 t1 = mul2(y, c[i]), t2 = mul2(partner, s[i]);
      z.v[i] = l < 4 ? make_float2(__fsub_rn(t1.x, t2.x), __fsub_rn(t1.y, t2.y)) : add2(t1, t2);
    }
    return z;
  }
}

template <typename TE>
__device__ __forceinline__ Frag norm_rope_frag(const Frag& x, int l, const Frag& w, const NormRopeArgs& a, int pos,
                                               int L, float* r_out) {
  return norm_rope_frag_w<TE>(x, l, w, a.eps, rope_words<TE>(a, pos, L, l), r_out);
}

// Rows [0, n) of a staged region starting at local position p0, normalised and
// rotated in place by the CTA's row groups.  (Fetching each iteration's table
// words during the iteration before measured slower in both fused kernels.)
// The trip count is the same for
// every row group (the helpers shuffle across the whole warp): groups past the
// end recompute row n - 1 and store nothing.
template <typename TE, int P>
__device__ __forceinline__ void norm_rope_smem_rows(uint8_t* base, int n, int p0, int grp, int l, const Frag& w,
                                                    const NormRopeArgs& a, int L) {
  for (int x0 = 0; x0 < n; x0 += kGroups) {
    const int x = x0 + grp < n ? x0 + grp : n - 1;
    uint8_t* row = base + x * P;
    const Frag z = norm_rope_frag<TE>(FragIO<TE>::load(row, l), l, w, a, p0 + x, L, nullptr);
    __syncwarp();
    if (x0 + grp < n) {
      if constexpr (sizeof(TE) == 2) {
        *reinterpret_cast<uint4*>(row + l * 16) = FragIO<TE>::pack(z);
      } else {
        *reinterpret_cast<float4*>(row + l * 32) = make_float4(z.v[0].x, z.v[0].y, z.v[1].x, z.v[1].y);
        *reinterpret_cast<float4*>(row + l * 32 + 16) = make_float4(z.v[2].x, z.v[2].y, z.v[3].x, z.v[3].y);
      }
    }
  }
}

// Backward of norm_rope_frag for one row: from dz (gradient of the rotated
// output, fp32) and the raw row x with its rsqrt r, returns dx and, if acc,
// adds the row's weight-gradient terms g * x * r to dw.  Every lane of the warp
// must call it (shuffles), whatever acc is.  g = RoPE transpose of dz:
//   g_j = dz_j c_j + dz_{j+32} s_j,   g_{j+32} = dz_{j+32} c_j - dz_j s_j,
//   dx  = r (g w) - x r^3 sum(g w x) / 64.
template <typename TE>
__device__ __forceinline__ Frag norm_rope_grad_w(const Frag& dz, const Frag& x, float r, int l, const Frag& w,
                                                 const RopeWords<TE>& rw, Frag& dw, bool acc) {
  const unsigned full = 0xffffffffu;
  const Frag c = FragIO<TE>::from_words(rw.c), s = FragIO<TE>::from_words(rw.s);
  const float sg = l < 4 ? 1.f : -1.f;
  const float2 rr = make_float2(r, r);
  Frag u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 partner = make_float2(__shfl_xor_sync(full, dz.v[i].x, 4), __shfl_xor_sync(full, dz.v[i].y, 4));
    const float2 g = fma2(make_float2(sg * partner.x, sg * partner.y), s.v[i], mul2(dz.v[i], c.v[i]));
    if (acc) dw.v[i] = fma2(g, mul2(x.v[i], rr), dw.v[i]);
    u.v[i] = mul2(g, w.v[i]);
  }
  const float k3 = r * r * r * nr_row_dot(u, x) * (1.f / 64.f);
  const float2 kk = make_float2(-k3, -k3);
  Frag dx;
#pragma unroll
  for (int i = 0; i < 4; ++i) dx.v[i] = fma2(x.v[i], kk, mul2(u.v[i], rr));
  return dx;
}

template <typename TE>
__device__ __forceinline__ Frag norm_rope_grad(const Frag& dz, const Frag& x, float r, int l, const Frag& w,
                                               const NormRopeArgs& a, int pos, int L, Frag& dw, bool acc) {
  return norm_rope_grad_w<TE>(dz, x, r, l, w, rope_words<TE>(a, pos, L, l), dw, acc);
}

// Per-CTA weight-gradient partials: the 16 row groups' fp32 sums (q then k) go
// through shared memory `scratch` (2 * 16 * 64 floats) and one row of
// [2, 64] per CTA is written in a fixed order.
__device__ __forceinline__ void nr_write_partials(float* partial, float* scratch, const Frag& dwq, const Frag& dwk,
                                                  int grp, int l) {
  float* sq = scratch + grp * 64 + 8 * l;
  float* sk = scratch + 16 * 64 + grp * 64 + 8 * l;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sq[2 * i] = dwq.v[i].x;
    sq[2 * i + 1] = dwq.v[i].y;
    sk[2 * i] = dwk.v[i].x;
    sk[2 * i + 1] = dwk.v[i].y;
  }
  __syncthreads();
  const int t = threadIdx.x;  // 128 threads: column t of [q 0..63 | k 0..63]
  const float* col = scratch + (t < 64 ? t : 16 * 64 + (t - 64));
  float sum = 0.f;
#pragma unroll
  for (int g = 0; g < 16; ++g) sum += col[g * 64];
  partial[(long long)blockIdx.x * 128 + t] = sum;
}

// --------------------------------------------------------------------------
// Forward
// --------------------------------------------------------------------------

// Source-set shapes of the forward: 0 = flags read at run time, 1 = {0, 1},
// 2 = {0, 2}, 3 = {0, 1, 2, d} with d >= TILE (own far tile), 4 = {0, 1, 2, d}
// with d < TILE (one window).
// NR: q and k arrive raw; each row is RMS-normalised and rotated on the way in
// (Q rows in registers, staged K rows once per CTA in shared memory).
template <typename TE, int LPR, bool TMA, int SHAPE, typename Maps = FwdMaps, bool NR = false>
__global__ void __launch_bounds__(kThreads) sbda_fwd_v2_kernel(const __grid_constant__ Maps maps,
                                                               const FwdV2Params p) {
  grid_dependency_sync();  // before any global memory access
  static_assert(!NR || (TMA && LPR == 8), "norm+RoPE is fused for the copy-engine path, 8 lanes per row");
  constexpr int T = v2_tile(LPR);
  constexpr int P = LPR * FragIO<TE>::kLaneBytes;
  extern __shared__ __align__(128) uint8_t smem[];
  const V2Geometry& g = p.g;
  const int tid = threadIdx.x;
  const int grp = tid / LPR, l = tid % LPR;

  int bid = blockIdx.x;
  const int h = bid % p.H;
  bid /= p.H;
  const int t = chain_tile_v2(bid % g.nT, g.R, g.A, g.rem);
  const int b = bid / g.nT;
  const int i0 = t * T;
  const int hk = h / p.G;  // kv head of query head h (grouped-query attention; G = 1 for MHA)
  const bool has1 = SHAPE == 0 ? g.has1 != 0 : (SHAPE == 1 || SHAPE >= 3);
  const bool has2 = SHAPE == 0 ? g.has2 != 0 : SHAPE >= 2;
  const bool far = SHAPE == 0 ? g.has_far != 0 : SHAPE >= 3;
  const bool has0 = SHAPE == 0 ? g.has0 != 0 : true;

  // The copy-engine path reads each group's Q rows straight into registers
  // (no Q tile in shared memory: more CTAs per SM); the generic path stages Q.
  // K/V rows [i0 - lead, i0 + T): lead = 2 (offsets 1, 2), or d when the far
  // offset is shorter than a tile -- its sources then lie in the same window
  // (staged once, as a d-row box and the tile, both tile-aligned).  A far offset
  // of a tile or more gets its own tile [i0 - d, i0 - d + T).
  const bool near_far = SHAPE == 0 ? far && g.d < T : SHAPE == 4;
  const int lead = near_far ? g.d : 2;
  uint8_t* Qs = smem;
  uint8_t* Kn = smem + (TMA ? 0 : T * P);
  uint8_t* Vn = Kn + (T + lead) * P;
  uint8_t* Kf = near_far ? Kn : Vn + (T + lead) * P;  // row r = source of query r
  uint8_t* Vf = near_far ? Vn : Kf + T * P;
  uint64_t* bar = reinterpret_cast<uint64_t*>(Vn + (T + lead) * P + (far && !near_far ? 2 * T * P : 0));

  const int a = grp * 4;
  RowWords<TE> qw[4];
  RopeWords<TE> qrw[4];  // NR: table words of the group's Q rows
  if constexpr (TMA) {
    if (tid == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
      // Each box lies in one rank's shard: this rank's map at local rows, or
      // (shards) pick_map gives the owner's map and row.
      const int ig = p.sh.pos0 + i0;
      int c;
      mbar_arrive_expect_tx(bar, (uint32_t)((2 * (T + lead) + (far && !near_far ? 2 * T : 0)) * P));
      if (own_rows(maps.kT, p.sh, i0 - lead, i0 + T)) {
        tma_rows(Kn, own_map(maps.kH, p.sh), bar, p.slots_k, i0 - lead, hk, b);
        tma_rows(Vn, own_map(maps.vH, p.sh), bar, p.slots_v, i0 - lead, hk, b);
        tma_rows(Kn + lead * P, own_map(maps.kT, p.sh), bar, p.slots_k, i0, hk, b);
        tma_rows(Vn + lead * P, own_map(maps.vT, p.sh), bar, p.slots_v, i0, hk, b);
      } else {
        tma_rows(Kn, pick_map(maps.kH, p.sh, ig - lead, c), bar, p.slots_k, c, hk, b);
        tma_rows(Vn, pick_map(maps.vH, p.sh, ig - lead, c), bar, p.slots_v, c, hk, b);
        tma_rows(Kn + lead * P, pick_map(maps.kT, p.sh, ig, c), bar, p.slots_k, c, hk, b);
        tma_rows(Vn + lead * P, pick_map(maps.vT, p.sh, ig, c), bar, p.slots_v, c, hk, b);
      }
      if (far && !near_far) {
        if (own_rows(maps.kT, p.sh, i0 - g.d, i0 - g.d + T)) {
          tma_rows(Kf, own_map(maps.kT, p.sh), bar, p.slots_k, i0 - g.d, hk, b);
          tma_rows(Vf, own_map(maps.vT, p.sh), bar, p.slots_v, i0 - g.d, hk, b);
        } else {
          tma_rows(Kf, pick_map(maps.kT, p.sh, ig - g.d, c), bar, p.slots_k, c, hk, b);
          tma_rows(Vf, pick_map(maps.vT, p.sh, ig - g.d, c), bar, p.slots_v, c, hk, b);
        }
      }
    }
    // Q rows of this group (and, NR, their table words), in flight while the K/V copies land.
    const TE* qb = reinterpret_cast<const TE*>(p.q.ptr) + (long long)b * p.q.sb + (long long)h * p.q.sh;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int pos = i0 + a + i;
      qw[i] = load_row_words<TE>(qb + (long long)min(pos, p.L - 1) * p.q.sl, p.D, l, pos < p.L);
      if constexpr (NR) qrw[i] = rope_words<TE>(p.nq, pos, p.L, l);
    }
    const bool ok = mbar_wait_bounded(bar, 0);
    if (__syncthreads_or(!ok)) {
      fault_and_drain(p.status, bar, 0);
      return;
    }
    if constexpr (NR) {
      // Staged K rows, each once: the window [i0 - lead, i0 + T) and the far tile.
      const Frag wk = nr_weights(p.nk.w, l);
      norm_rope_smem_rows<TE, P>(Kn, T + lead, i0 - lead, grp, l, wk, p.nk, p.L);
      if (far && !near_far) norm_rope_smem_rows<TE, P>(Kf, T, i0 - g.d, grp, l, wk, p.nk, p.L);
      __syncthreads();
    }
  } else {
    constexpr int PE = P / sizeof(TE);
    generic_rows<TE>(Qs, p.q, b, h, i0, T, p.L, p.D, PE);
    generic_rows<TE>(Kn, p.k, b, hk, i0 - lead, T + lead, p.L, p.D, PE);
    generic_rows<TE>(Vn, p.v, b, hk, i0 - lead, T + lead, p.L, p.D, PE);
    if (far && !near_far) {
      generic_rows<TE>(Kf, p.k, b, hk, i0 - g.d, T, p.L, p.D, PE);
      generic_rows<TE>(Vf, p.v, b, hk, i0 - g.d, T, p.L, p.D, PE);
    }
    __syncthreads();
  }

  const float c1 = p.scale * kLog2e;
  TE* out = reinterpret_cast<TE*>(const_cast<void*>(p.out.ptr)) + (long long)b * p.out.sb +
            (long long)h * p.out.sh;
  float* lse = p.lse + ((long long)b * p.H + h) * p.L;
  // Source owned by this lane pair in the reduce-scatter softmax (8 lanes per row).
  const int src_k = (l >> 1) & 3;
  const bool src_has = src_k == 0 ? has0 : (src_k == 1 ? has1 : (src_k == 2 ? has2 : far));
  const int src_off = src_k == 0 ? 0 : (src_k == 1 ? 1 : (src_k == 2 ? 2 : g.d));
  Frag k1 = FragIO<TE>::load(Kn + (a + lead - 1) * P, l), k2 = FragIO<TE>::load(Kn + (a + lead - 2) * P, l);
  Frag v1 = FragIO<TE>::load(Vn + (a + lead - 1) * P, l), v2 = FragIO<TE>::load(Vn + (a + lead - 2) * P, l);
  Frag wq;
  if constexpr (NR) wq = nr_weights(p.nq.w, l);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = a + i, pos = i0 + r;
    const int pg = p.sh.pos0 + pos;  // global position: source masks
    Frag q = TMA ? FragIO<TE>::from_words(qw[i].w) : FragIO<TE>::load(Qs + r * P, l);
    if constexpr (NR) q = norm_rope_frag_w<TE>(q, l, wq, p.nq.eps, qrw[i], nullptr);
    const Frag k0 = FragIO<TE>::load(Kn + (r + lead) * P, l);
    const Frag v0 = FragIO<TE>::load(Vn + (r + lead) * P, l);
    if constexpr (LPR == 8) {
      // Reduce-scatter softmax: lanes 2k and 2k + 1 of the group hold the score of
      // source k; max, exponent and sum are formed once per source.
      float x[4];
      x[0] = frag_dot(q, k0);
      x[1] = has1 ? frag_dot(q, k1) : 0.f;
      x[2] = has2 ? frag_dot(q, k2) : 0.f;
      x[3] = 0.f;
      Frag vf;
      if (far) {
        const Frag kf = FragIO<TE>::load(Kf + r * P, l);
        x[3] = frag_dot(q, kf);
        vf = FragIO<TE>::load(Vf + r * P, l);
      }
      const unsigned full = 0xffffffffu;
      const float val = group8_reduce_scatter4(x, l);
      const bool live = src_has && pg >= src_off;
      const float sc = live ? val * c1 : -INFINITY;  // log2 units
      float m = fmaxf(sc, __shfl_xor_sync(full, sc, 2));
      m = fmaxf(m, __shfl_xor_sync(full, m, 4));
      const bool any = m != -INFINITY;
      const float e = live ? fast_exp2(sc - m) : 0.f;
      float sum = e + __shfl_xor_sync(full, e, 2);
      sum += __shfl_xor_sync(full, sum, 4);
      const float inv = any ? __frcp_rn(sum) : 0.f;
      const float w = e * inv;
      const float w0 = __shfl_sync(full, w, 0, 8), w1 = __shfl_sync(full, w, 2, 8);
      const float w2 = __shfl_sync(full, w, 4, 8), wf = __shfl_sync(full, w, 6, 8);
      Frag o = frag_mul(w0, v0);
      if (has1) frag_axpy(o, w1, v1);
      if (has2) frag_axpy(o, w2, v2);
      if (far) frag_axpy(o, wf, vf);
      if (pos < p.L) {
        store_frag<TE, TMA>(out + (long long)pos * p.out.sl, p.out.sd, p.D, l, o);
        if (l == 0) lse[pos] = any ? (m + __log2f(sum)) * kLn2 : -INFINITY;
      }
      k2 = k1;
      k1 = k0;
      v2 = v1;
      v1 = v0;
      continue;
    }
    float s0 = lane_group_sum<LPR>(frag_dot(q, k0));
    float s1 = has1 ? lane_group_sum<LPR>(frag_dot(q, k1)) : 0.f;
    float s2 = has2 ? lane_group_sum<LPR>(frag_dot(q, k2)) : 0.f;
    float sf = 0.f;
    Frag vf;
    if (far) {
      const Frag kf = FragIO<TE>::load(Kf + r * P, l);
      sf = lane_group_sum<LPR>(frag_dot(q, kf));
      vf = FragIO<TE>::load(Vf + r * P, l);
    }
    // scores in log2 units: s * scale * log2(e)
    const bool u0 = has0, u1 = has1 && pg >= 1, u2 = has2 && pg >= 2, uf = far && pg >= g.d;
    s0 = u0 ? s0 * c1 : -INFINITY;
    s1 = u1 ? s1 * c1 : -INFINITY;
    s2 = u2 ? s2 * c1 : -INFINITY;
    sf = uf ? sf * c1 : -INFINITY;
    const float m = fmaxf(fmaxf(s0, s1), fmaxf(s2, sf));
    const bool any = m != -INFINITY;
    const float e0 = u0 ? fast_exp2(s0 - m) : 0.f, e1 = u1 ? fast_exp2(s1 - m) : 0.f;
    const float e2 = u2 ? fast_exp2(s2 - m) : 0.f, ef = uf ? fast_exp2(sf - m) : 0.f;
    const float sum = (e0 + e1) + (e2 + ef);
    const float inv = any ? __frcp_rn(sum) : 0.f;
    Frag o = frag_mul(e0 * inv, v0);
    if (has1) frag_axpy(o, e1 * inv, v1);
    if (has2) frag_axpy(o, e2 * inv, v2);
    if (far) frag_axpy(o, ef * inv, vf);
    if (pos < p.L) {
      store_frag<TE, TMA>(out + (long long)pos * p.out.sl, p.out.sd, p.D, l, o);
      if (l == 0) lse[pos] = any ? (m + __log2f(sum)) * kLn2 : -INFINITY;
    }
    k2 = k1;
    k1 = k0;
    v2 = v1;
    v1 = v0;
  }
}

// --------------------------------------------------------------------------
// Backward
// --------------------------------------------------------------------------

// Issues the copies of one K/V slot: rows [p0, p0 + halo + T + halo) of the
// call's rows (p0 local).  Every box lies in one rank's shard (shards are tile
// multiples, halos are shorter than a tile): pick_map gives its map and row.
template <typename TE, int T, int P, typename Maps>
__device__ __forceinline__ void tma_kv_slot(const Maps& maps, const BwdV2Params& p, uint64_t* bar,
                                            uint8_t* K, uint8_t* V, int p0, int halo, int h, int b) {
  if (own_rows(maps.kT, p.sh, p0, p0 + 2 * halo + T)) {
    tma_rows(K, own_map(maps.kH, p.sh), bar, p.slots_k, p0, h, b);
    tma_rows(V, own_map(maps.vH, p.sh), bar, p.slots_v, p0, h, b);
    tma_rows(K + halo * P, own_map(maps.kT, p.sh), bar, p.slots_k, p0 + halo, h, b);
    tma_rows(V + halo * P, own_map(maps.vT, p.sh), bar, p.slots_v, p0 + halo, h, b);
    tma_rows(K + (halo + T) * P, own_map(maps.kH, p.sh), bar, p.slots_k, p0 + halo + T, h, b);
    tma_rows(V + (halo + T) * P, own_map(maps.vH, p.sh), bar, p.slots_v, p0 + halo + T, h, b);
    return;
  }
  const int g0 = p.sh.pos0 + p0;
  int c;
  tma_rows(K, pick_map(maps.kH, p.sh, g0, c), bar, p.slots_k, c, h, b);
  tma_rows(V, pick_map(maps.vH, p.sh, g0, c), bar, p.slots_v, c, h, b);
  tma_rows(K + halo * P, pick_map(maps.kT, p.sh, g0 + halo, c), bar, p.slots_k, c, h, b);
  tma_rows(V + halo * P, pick_map(maps.vT, p.sh, g0 + halo, c), bar, p.slots_v, c, h, b);
  tma_rows(K + (halo + T) * P, pick_map(maps.kH, p.sh, g0 + halo + T, c), bar, p.slots_k, c, h, b);
  tma_rows(V + (halo + T) * P, pick_map(maps.vH, p.sh, g0 + halo + T, c), bar, p.slots_v, c, h, b);
}

template <typename TE, int T, int P, typename Maps>
__device__ __forceinline__ void tma_qd_slot(const Maps& maps, const BwdV2Params& p, uint64_t* bar,
                                            uint8_t* Q, uint8_t* Dd, int j0, int halo, int h, int b) {
  if (own_rows(maps.qT, p.sh, j0, j0 + T + halo)) {
    tma_rows(Q, own_map(maps.qT, p.sh), bar, p.slots_q, j0, h, b);
    tma_rows(Dd, own_map(maps.dT, p.sh), bar, p.slots_d, j0, h, b);
    tma_rows(Q + T * P, own_map(maps.qH, p.sh), bar, p.slots_q, j0 + T, h, b);
    tma_rows(Dd + T * P, own_map(maps.dH, p.sh), bar, p.slots_d, j0 + T, h, b);
    return;
  }
  const int g0 = p.sh.pos0 + j0;
  int c;
  tma_rows(Q, pick_map(maps.qT, p.sh, g0, c), bar, p.slots_q, c, h, b);
  tma_rows(Dd, pick_map(maps.dT, p.sh, g0, c), bar, p.slots_d, c, h, b);
  tma_rows(Q + T * P, pick_map(maps.qH, p.sh, g0 + T, c), bar, p.slots_q, c, h, b);
  tma_rows(Dd + T * P, pick_map(maps.dH, p.sh, g0 + T, c), bar, p.slots_d, c, h, b);
}

// LSE rows of a Q/dO slot (the tile and the consumers past it).  One GPU: one
// box of lse_box rows.  Shards: the tile's rows from this rank and the halo
// rows from their owner (past the sequence end: this rank's map out of range,
// zero-filled); both boxes start at tile-aligned rows.
template <int T>
__device__ __forceinline__ void tma_lse_slot(const BwdMaps& maps, const BwdV2Params& p, uint64_t* bar,
                                             float* dst, int j0, int halo, int row) {
  tma_2d(dst, &maps.lseT, bar, j0, row);
}
template <int T>
__device__ __forceinline__ void tma_lse_slot(const ShardBwdMaps& maps, const BwdV2Params& p, uint64_t* bar,
                                             float* dst, int j0, int halo, int row) {
  // The halo box may run past the consumers used (rows T + halo.. are padding).
  if (own_rows(maps.lseT, p.sh, j0, j0 + T + halo)) {
    tma_2d(dst, own_map(maps.lseT, p.sh), bar, j0, row);
    tma_2d(dst + T, own_map(maps.lseH, p.sh), bar, j0 + T, row);
    return;
  }
  const int g0 = p.sh.pos0 + j0;
  int c;
  const CUtensorMap* m = pick_map(maps.lseT, p.sh, g0, c);
  tma_2d(dst, m, bar, c, row);
  m = pick_map(maps.lseH, p.sh, g0 + T, c);
  tma_2d(dst + T, m, bar, c, row);
}

// Source-set shapes the backward is compiled for.  0 reads the flags at run
// time; the others fix them so the per-row code is straight-line:
//   1: {0, 1} (SBDA layer 1)          2: {0, 2} (SBDA layer 2)
//   3: {0, 1, 2, d}, d < TILE, d % 4 == 0 (local carry)
//   4: {0, 1, 2, d}, d % TILE == 0 (chain walk)
//   5: {0, 1, 2, d}, d < TILE (local)
template <int SHAPE>
struct BwdShape {
  static constexpr bool kGeneric = SHAPE == 0;
  static constexpr bool kHas1 = SHAPE == 1 || SHAPE >= 3;
  static constexpr bool kHas2 = SHAPE >= 2;
  static constexpr bool kFar = SHAPE >= 3;
  static constexpr bool kChain = SHAPE == 4;
  static constexpr bool kLocalCarry = SHAPE == 3;
};

// NR: q and k arrive raw and dq, dk leave raw.  Staged K rows are normalised
// and rotated in place once per staging (a chain walk's far tile is the next
// step's near tile); each Q row by the row group that consumes it in phase 1,
// which writes it back for phase 2.  dQ gets the norm+RoPE Jacobian in phase
// 1 (raw q still in registers), dK in phase 2 (raw k re-read from global,
// usually an L2 hit); the norm-weight gradients are summed per CTA into
// p.dw_partial.
// TO: element type of the dK/dV rows written.  TE (the input type) writes the
// final gradients; float writes one query head's fp32 partials of grouped-query
// attention (K/V rows from kv head h / G), summed per kv head afterwards.
template <typename TE, int LPR, bool TMA, int SHAPE, typename Maps = BwdMaps, bool NR = false, typename TO = TE>
__global__ void __launch_bounds__(kThreads, NR ? 2 : 3) sbda_bwd_v2_kernel(const __grid_constant__ Maps maps,
                                                                  const BwdV2Params p) {
  grid_dependency_sync();  // before any global memory access
  static_assert(!NR || (TMA && LPR == 8), "norm+RoPE is fused for the copy-engine path, 8 lanes per row");
  constexpr int T = v2_tile(LPR);
  constexpr int P = LPR * FragIO<TE>::kLaneBytes;
  constexpr int GROUPS = kThreads / LPR;
  constexpr int GPW = 32 / LPR;  // row groups per warp
  using Sh = BwdShape<SHAPE>;
  extern __shared__ __align__(128) uint8_t smem[];
  const V2Geometry& g = p.g;
  const int tid = threadIdx.x;
  const int grp = tid / LPR, l = tid % LPR;
  const bool has0 = Sh::kGeneric ? g.has0 != 0 : true;
  const bool has1 = Sh::kGeneric ? g.has1 != 0 : Sh::kHas1;
  const bool has2 = Sh::kGeneric ? g.has2 != 0 : Sh::kHas2;
  const bool far = Sh::kGeneric ? g.has_far != 0 : Sh::kFar;
  const bool chain = Sh::kGeneric ? g.mode == 0 : Sh::kChain;
  const bool lc = Sh::kGeneric ? g.mode == 2 : Sh::kLocalCarry;
  const int Hc = (Sh::kGeneric || SHAPE == 5) ? g.halo : 2;  // consumer rows past the tile
  const int d = g.d;
  // Source owned by this lane in the reduce-scatter softmax (8 lanes per row).
  const int src_k = l & 3;
  const bool src_has = src_k == 0 ? has0 : (src_k == 1 ? has1 : (src_k == 2 ? has2 : far));
  const int src_off = src_k == 0 ? 0 : (src_k == 1 ? 1 : (src_k == 2 ? 2 : d));
  const int lead = lc ? d : Hc;                  // K/V rows of a near slot before the tile
  const int KVR = lc ? T + d : T + 2 * Hc;       // rows of a K/V slot
  const int QDR = T + Hc;                        // rows of a Q/dO slot
  const int nkv = chain ? 2 : 1;

  // ---- Work assignment: a walk of tiles for this CTA. ----
  // Heads vary fastest across consecutive CTAs: the rows of all heads of a
  // position share DRAM pages and L2 lines in the [B, L, H, D] layout, so
  // the heads of one walk segment run side by side.  Chains (residues r) vary
  // next, before segments: neighbouring chains then walk side by side, and the
  // 2-row halos a step reads from the adjacent tiles (another chain's) are in L2.
  int bid = blockIdx.x;
  int b, h, t_first, n_steps, stride, pre;
  h = bid % p.H;
  bid /= p.H;
  if (chain) {
    const int r = bid % g.chains;
    bid /= g.chains;
    const int s = bid % g.segs;
    b = bid / g.segs;
    const int A_r = (g.nT - 1 - r) / g.R + 1;
    const int a_lo = s * g.seg;
    if (a_lo >= A_r) {
      if constexpr (NR) p.dw_partial[(long long)blockIdx.x * 128 + tid] = 0.f;
      return;
    }
    const int a_hi = min(a_lo + g.seg, A_r) - 1;
    // The tile above the segment may be on the next rank's shard (sharded calls).
    pre = p.sh.pos0 / T + (a_hi + 1) * g.R + r < (p.sh.total_len + T - 1) / T;
    t_first = (a_hi + pre) * g.R + r;
    n_steps = a_hi - a_lo + 1 + pre;
    stride = g.R;
  } else {
    const int s = bid % g.segs;
    b = bid / g.segs;
    const int lo = s * g.seg;
    if (lo >= g.nT) {
      if constexpr (NR) p.dw_partial[(long long)blockIdx.x * 128 + tid] = 0.f;
      return;
    }
    const int hi = min(lo + g.seg, g.nT) - 1;
    pre = lc && p.sh.pos0 / T + hi + 1 < (p.sh.total_len + T - 1) / T;
    t_first = hi + pre;
    n_steps = hi - lo + 1 + pre;
    stride = 1;
  }

  const int hk = h / p.G;                        // kv head of query head h (1 = MHA: hk = h)
  uint8_t* KVbase = smem;                        // nkv slots of [K rows][V rows]
  uint8_t* QDbase = KVbase + nkv * 2 * KVR * P;  // 2 slots of [Q rows][dO rows]
  // Softmax records, a ring of 2T consumers: (p0, ds0, p1, ds1) (p2, ds2, pf, dsf)
  // per consumer, ds already scaled by head_dim^-0.5.  Consumer c of step s sits
  // at ring row (s * T + c) mod 2T, so rows T.. of a step are rows 0.. of the
  // step before.  Every 4 rows carry 16 bytes of padding: the row groups of a
  // warp (4 rows apart) then start on different banks.
  float* E = reinterpret_cast<float*>(QDbase + 2 * 2 * QDR * P);
  // Two LSE slots of lse_box fp32 rows each (128-byte multiples), 128-byte aligned after E.
  float* LSEs = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(E + v2_ring_floats(T)) + 127) & ~uintptr_t(127));
  uint64_t* bars = reinterpret_cast<uint64_t*>(LSEs + 2 * p.lse_box);
  auto kslot = [&](int s) { return KVbase + s * 2 * KVR * P; };
  auto vslot = [&](int s) { return KVbase + s * 2 * KVR * P + KVR * P; };
  auto qslot = [&](int s) { return QDbase + s * 2 * QDR * P; };
  auto dslot = [&](int s) { return QDbase + s * 2 * QDR * P + QDR * P; };

  // Copies of step i: the Q/dO batch (issued a whole step ahead) and the K/V
  // batch (issued once phase 1 of the previous step has released its slot).
  // Each batch is one arrival on the step's barrier (count 2).
  auto issue_qd = [&](int i) {
    const int j0 = (t_first - i * stride) * T;
    if constexpr (TMA) {
      uint64_t* bar = bars + (i & 1);
      mbar_arrive_expect_tx(bar, (uint32_t)(2 * QDR * P + (p.lse_tma ? p.lse_tx : 0)));
      tma_qd_slot<TE, T, P>(maps, p, bar, qslot(i & 1), dslot(i & 1), j0, Hc, h, b);
      if (p.lse_tma) tma_lse_slot<T>(maps, p, bar, LSEs + (i & 1) * p.lse_box, j0, Hc, b * p.H + h);
    } else {
      constexpr int PE = P / sizeof(TE);
      generic_rows<TE>(qslot(i & 1), p.q, b, h, j0, QDR, p.L, p.D, PE);
      generic_rows<TE>(dslot(i & 1), p.dout, b, h, j0, QDR, p.L, p.D, PE);
    }
  };
  auto issue_kv = [&](int i) {
    const int j0 = (t_first - i * stride) * T;
    // chain: step 0 stages its near slot 0 and far slot 1; step i > 0 stages
    // only its far tile, into slot (i + 1) & 1 (its near tile is step i-1's far).
    const int first = chain ? (i == 0 ? 0 : 1) : 0;
    if constexpr (TMA) {
      uint64_t* bar = bars + (i & 1);
      mbar_arrive_expect_tx(bar, (uint32_t)((chain && i == 0 ? 2 : 1) * 2 * KVR * P));
      if (lc && own_rows(maps.kT, p.sh, j0 - d, j0 + T)) {  // rows [j0 - d, j0 + T): a d-row box, then the tile
        tma_rows(kslot(0), own_map(maps.kH, p.sh), bar, p.slots_k, j0 - d, hk, b);
        tma_rows(vslot(0), own_map(maps.vH, p.sh), bar, p.slots_v, j0 - d, hk, b);
        tma_rows(kslot(0) + d * P, own_map(maps.kT, p.sh), bar, p.slots_k, j0, hk, b);
        tma_rows(vslot(0) + d * P, own_map(maps.vT, p.sh), bar, p.slots_v, j0, hk, b);
      } else if (lc) {
        const int jg = p.sh.pos0 + j0;
        int c;
        tma_rows(kslot(0), pick_map(maps.kH, p.sh, jg - d, c), bar, p.slots_k, c, hk, b);
        tma_rows(vslot(0), pick_map(maps.vH, p.sh, jg - d, c), bar, p.slots_v, c, hk, b);
        tma_rows(kslot(0) + d * P, pick_map(maps.kT, p.sh, jg, c), bar, p.slots_k, c, hk, b);
        tma_rows(vslot(0) + d * P, pick_map(maps.vT, p.sh, jg, c), bar, p.slots_v, c, hk, b);
      } else {
        for (int part = first; part < (chain ? 2 : 1); ++part) {
          const int slot = chain ? ((i + part) & 1) : 0;
          const int p0 = part == 0 ? j0 - Hc : j0 - d - Hc;
          tma_kv_slot<TE, T, P>(maps, p, bar, kslot(slot), vslot(slot), p0, Hc, hk, b);
        }
      }
    } else {
      constexpr int PE = P / sizeof(TE);
      for (int part = first; part < (chain ? 2 : 1); ++part) {
        const int slot = chain ? ((i + part) & 1) : 0;
        const int p0 = part == 0 ? j0 - lead : j0 - d - Hc;
        generic_rows<TE>(kslot(slot), p.k, b, hk, p0, KVR, p.L, p.D, PE);
        generic_rows<TE>(vslot(slot), p.v, b, hk, p0, KVR, p.L, p.D, PE);
      }
    }
  };

  if constexpr (TMA) {
    if (tid == 0) {
      mbar_init(bars, 2);
      mbar_init(bars + 1, 2);
      fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
      issue_qd(0);
      issue_kv(0);
    }
  }

  const float scale = p.scale;
  const float c1 = scale * kLog2e;  // exp(a * scale - lse) = 2^(a * c1 - lse * log2 e)
  const long long bh = (long long)b * p.H + h;
  // log2-scaled LSE of consumer row j0 + c (local rows; past the shard end it is
  // the next rank's row), 0 past the sequence.
  auto lse_row = [&](int j0, int c) -> float {
    const int qg = p.sh.pos0 + j0 + c;
    return qg < p.sh.total_len ? lse_at(p.sh, bh, qg) * kLog2e : 0.f;
  };
  TE* dq = reinterpret_cast<TE*>(const_cast<void*>(p.dq.ptr)) + (long long)b * p.dq.sb + (long long)h * p.dq.sh;
  TO* dk = reinterpret_cast<TO*>(const_cast<void*>(p.dk.ptr)) + (long long)b * p.dk.sb + (long long)h * p.dk.sh;
  TO* dv = reinterpret_cast<TO*>(const_cast<void*>(p.dv.ptr)) + (long long)b * p.dv.sb + (long long)h * p.dv.sh;

  // Far-edge dK/dV contributions carried to the next tile of a chain walk.
  Frag carry_k[4], carry_v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) carry_k[i] = carry_v[i] = frag_zero();
  // NR: this lane's norm-weight gradient sums (q, k) over the rows it finishes.
  Frag dwq = frag_zero(), dwk = frag_zero();

  // One step of the walk.  The carry-only "pre" tile is a separate instance
  // (PreTag = true_type), so the steady-state loop has no per-step pre tests.
  // Returns false when a copy wait expired; the CTA then stops.
  auto run_step = [&](const int step, auto pre_tag) -> bool {
    constexpr bool is_pre = decltype(pre_tag)::value;
    const int t = t_first - step * stride;
    const int j0 = t * T;
    if constexpr (TMA) {
      if (tid == 0 && step + 1 < n_steps) issue_qd(step + 1);
      const bool ok = mbar_wait_bounded(bars + (step & 1), (step >> 1) & 1);
      if (__syncthreads_or(!ok)) {
        fault_and_drain(p.status, bars + (step & 1), (step >> 1) & 1);
        return false;
      }
    } else {
      issue_qd(step);
      issue_kv(step);
      __syncthreads();
    }
    if constexpr (NR) {
      // K rows staged for this step, each once: a chain walk stages its far slot
      // every step (both slots at its first step); other walks restage their slot.
      const Frag wk = nr_weights(p.nk.w, l);
      for (int part = chain && step > 0 ? 1 : 0; part < (chain ? 2 : 1); ++part) {
        const int slot = chain ? ((step + part) & 1) : 0;
        const int p0 = lc ? j0 - d : (part == 0 ? j0 - Hc : j0 - d - Hc);
        norm_rope_smem_rows<TE, P>(kslot(slot), KVR, p0, grp, l, wk, p.nk, p.L);
      }
      __syncthreads();
    }
    const int ns = chain ? (step & 1) : 0;
    const uint8_t* KN = kslot(ns);
    const uint8_t* VN = vslot(ns);
    const uint8_t* KF = chain ? kslot(ns ^ 1) : KN;
    const uint8_t* VF = chain ? vslot(ns ^ 1) : VN;
    const int fidx = chain ? Hc : lead - d;  // far source row of consumer c = c + fidx
    const uint8_t* Qs = qslot(step & 1);
    const uint8_t* Ds = dslot(step & 1);
    const int ebase = (step & 1) * T;
    // Record of consumer c: ring row x = (ebase + c) mod 2T at float x * 8 + (x / 4) * 4,
    // i.e. 9 * x for x a multiple of 4 and 8 floats further per row after it.
    auto erec = [&](int c) -> float* {
      const int x = (ebase + c) & (2 * T - 1);
      return E + x * 8 + (x >> 2) * 4;
    };
    auto egroup = [&](int c4) -> float* { return E + 9 * ((ebase + c4) & (2 * T - 1)); };  // c4 % 4 == 0

    // ---- Phase 1: softmax terms of every consumer, dQ of own queries. ----
    auto consume = [&](int c, bool act, float* erow, const Frag& k0, const Frag& v0, const Frag& k1,
                       const Frag& v1, const Frag& k2, const Frag& v2, float lq2) {
      const int q = j0 + c;             // local row (dQ store)
      const int qg = p.sh.pos0 + q;     // global position (masks)
      const Frag qx = FragIO<TE>::load(Qs + c * P, l);  // raw q when NR
      Frag qf = qx;
      float rq = 0.f;
      if constexpr (NR) {
        // Normalise this consumer's row; phase 2 reads it back from the slot.
        qf = norm_rope_frag<TE>(qx, l, nr_weights(p.nq.w, l), p.nq, q, p.L, &rq);
        __syncwarp();
        if (act) {
          uint8_t* row = const_cast<uint8_t*>(Qs) + c * P;
          if constexpr (sizeof(TE) == 2) {
            *reinterpret_cast<uint4*>(row + l * 16) = FragIO<TE>::pack(qf);
          } else {
            *reinterpret_cast<float4*>(row + l * 32) = make_float4(qf.v[0].x, qf.v[0].y, qf.v[1].x, qf.v[1].y);
            *reinterpret_cast<float4*>(row + l * 32 + 16) = make_float4(qf.v[2].x, qf.v[2].y, qf.v[3].x, qf.v[3].y);
          }
        }
      }
      const Frag df = FragIO<TE>::load(Ds + c * P, l);
      if constexpr (LPR == 8) {
        // Reduce-scatter softmax: after the exchange lanes l and l ^ 4 both hold q.k
        // and dO.v of source l & 3 and form its p and ds (the same values on both),
        // so p needs no exchange between the score lanes and the dO.v lanes.
        float x[8];
        x[0] = frag_dot(qf, k0);
        x[4] = frag_dot(df, v0);
        x[1] = has1 ? frag_dot(qf, k1) : 0.f;
        x[5] = has1 ? frag_dot(df, v1) : 0.f;
        x[2] = has2 ? frag_dot(qf, k2) : 0.f;
        x[6] = has2 ? frag_dot(df, v2) : 0.f;
        x[3] = x[7] = 0.f;
        Frag kf;
        if (far) {
          kf = FragIO<TE>::load(KF + (c + fidx) * P, l);
          const Frag vf = FragIO<TE>::load(VF + (c + fidx) * P, l);
          x[3] = frag_dot(qf, kf);
          x[7] = frag_dot(df, vf);
        }
        const unsigned full = 0xffffffffu;
        const float2 ab = group8_reduce_scatter_pairs(x, l);  // (q.k, dO.v) of source l & 3
        const bool inr = qg < p.sh.total_len;
        const bool live = src_has && inr && qg >= src_off;
        const float ps = live ? fast_exp2(fmaf(ab.x, c1, -lq2)) : 0.f;
        const float t = ps * ab.y;
        float delta = t + __shfl_xor_sync(full, t, 1);
        delta += __shfl_xor_sync(full, delta, 2);
        const float ds = ps * (ab.y - delta) * scale;
        const float d0 = __shfl_sync(full, ds, 0, 8), d1 = __shfl_sync(full, ds, 1, 8);
        const float d2 = __shfl_sync(full, ds, 2, 8), dfw = __shfl_sync(full, ds, 3, 8);
        const bool store_q = act && c < T && inr && !is_pre;
        if constexpr (NR) {
          // dQ of the raw row: RoPE transpose and RMSNorm Jacobian (every lane shuffles).
          if (!is_pre) {
            Frag gq = frag_mul(d0, k0);
            if (has1) frag_axpy(gq, d1, k1);
            if (has2) frag_axpy(gq, d2, k2);
            if (far) frag_axpy(gq, dfw, kf);
            const Frag gx = norm_rope_grad<TE>(gq, qx, rq, l, nr_weights(p.nq.w, l), p.nq, q, p.L, dwq, store_q);
            if (store_q) store_frag<TE, TMA>(dq + (long long)q * p.dq.sl, p.dq.sd, p.D, l, gx);
          }
        } else if (store_q) {
          Frag gq = frag_mul(d0, k0);
          if (has1) frag_axpy(gq, d1, k1);
          if (has2) frag_axpy(gq, d2, k2);
          if (far) frag_axpy(gq, dfw, kf);
          store_frag<TE, TMA>(dq + (long long)q * p.dq.sl, p.dq.sd, p.D, l, gq);
        }
        if (act && l < 4) reinterpret_cast<float2*>(erow)[l] = make_float2(ps, ds);
        return;
      }
      const float a0 = lane_group_sum<LPR>(frag_dot(qf, k0));
      const float b0 = lane_group_sum<LPR>(frag_dot(df, v0));
      float a1 = 0.f, b1 = 0.f, a2 = 0.f, b2 = 0.f, af = 0.f, bf = 0.f;
      if (has1) {
        a1 = lane_group_sum<LPR>(frag_dot(qf, k1));
        b1 = lane_group_sum<LPR>(frag_dot(df, v1));
      }
      if (has2) {
        a2 = lane_group_sum<LPR>(frag_dot(qf, k2));
        b2 = lane_group_sum<LPR>(frag_dot(df, v2));
      }
      Frag kf;
      if (far) {
        kf = FragIO<TE>::load(KF + (c + fidx) * P, l);
        const Frag vf = FragIO<TE>::load(VF + (c + fidx) * P, l);
        af = lane_group_sum<LPR>(frag_dot(qf, kf));
        bf = lane_group_sum<LPR>(frag_dot(df, vf));
      }
      const bool inr = qg < p.sh.total_len;
      const bool u0 = has0 && inr, u1 = has1 && inr && qg >= 1, u2 = has2 && inr && qg >= 2;
      const bool uf = far && inr && qg >= d;
      const float p0 = u0 ? fast_exp2(fmaf(a0, c1, -lq2)) : 0.f;
      const float p1 = u1 ? fast_exp2(fmaf(a1, c1, -lq2)) : 0.f;
      const float p2 = u2 ? fast_exp2(fmaf(a2, c1, -lq2)) : 0.f;
      const float pf = uf ? fast_exp2(fmaf(af, c1, -lq2)) : 0.f;
      const float delta = fmaf(p0, b0, fmaf(p1, b1, fmaf(p2, b2, pf * bf)));
      const float d0 = p0 * (b0 - delta) * scale, d1 = p1 * (b1 - delta) * scale;
      const float d2 = p2 * (b2 - delta) * scale, dfw = pf * (bf - delta) * scale;
      if (act && c < T && inr && !is_pre) {
        Frag gq = frag_mul(d0, k0);
        if (has1) frag_axpy(gq, d1, k1);
        if (has2) frag_axpy(gq, d2, k2);
        if (far) frag_axpy(gq, dfw, kf);
        store_frag<TE, TMA>(dq + (long long)q * p.dq.sl, p.dq.sd, p.D, l, gq);
      }
      if (act && l == 0) {
        float4* e = reinterpret_cast<float4*>(erow);
        e[0] = make_float4(p0, d0, p1, d1);
        e[1] = make_float4(p2, d2, pf, dfw);
      }
    };

    {
      const int a = grp * 4;
      float lq[4];
      const float* ls = LSEs + (step & 1) * p.lse_box;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        lq[i] = (TMA && p.lse_tma) ? ls[a + i] * kLog2e : lse_row(j0, a + i);
      Frag k1 = FragIO<TE>::load(KN + (a + lead - 1) * P, l), k2 = FragIO<TE>::load(KN + (a + lead - 2) * P, l);
      Frag v1 = FragIO<TE>::load(VN + (a + lead - 1) * P, l), v2 = FragIO<TE>::load(VN + (a + lead - 2) * P, l);
      float* Eg = egroup(a);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = a + i;
        const Frag k0 = FragIO<TE>::load(KN + (c + lead) * P, l);
        const Frag v0 = FragIO<TE>::load(VN + (c + lead) * P, l);
        consume(c, true, Eg + 8 * i, k0, v0, k1, v1, k2, v2, lq[i]);
        k2 = k1;
        k1 = k0;
        v2 = v1;
        v1 = v0;
      }
    }
    // Consumers past the tile: runs of xr rows; warps with no live row skip.
    // A walk of consecutive tiles has them from the step before; in local carry
    // mode only their near sources are read, and the first step of a walk
    // without a pre tile starts at the sequence end, where they are empty.
    if (lc) {
      if (step == 0 && !pre && tid < 2 * 8) erec(T + (tid >> 3))[tid & 7] = 0.f;
    } else if (stride != 1 || step == 0) {
      const int xr = (Hc + GROUPS - 1) / GROUPS;
      const int warp_first = (tid >> 5) * GPW * xr;
      if (warp_first < Hc) {
        const int e0 = grp * xr;
        const int cbase = T + min(e0, Hc - 1);
        Frag k1 = FragIO<TE>::load(KN + (cbase + lead - 1) * P, l);
        Frag k2 = FragIO<TE>::load(KN + (cbase + lead - 2) * P, l);
        Frag v1 = FragIO<TE>::load(VN + (cbase + lead - 1) * P, l);
        Frag v2 = FragIO<TE>::load(VN + (cbase + lead - 2) * P, l);
#pragma unroll 1
        for (int i = 0; i < xr; ++i) {
          const bool act = e0 + i < Hc;
          const int c = act ? T + e0 + i : cbase;
          const float lq = (TMA && p.lse_tma) ? LSEs[(step & 1) * p.lse_box + c] * kLog2e
                                              : (act ? lse_row(j0, c) : 0.f);
          const Frag k0 = FragIO<TE>::load(KN + (c + lead) * P, l);
          const Frag v0 = FragIO<TE>::load(VN + (c + lead) * P, l);
          consume(c, act, erec(c), k0, v0, k1, v1, k2, v2, lq);
          k2 = k1;
          k1 = k0;
          v2 = v1;
          v1 = v0;
        }
      }
    }
    if constexpr (NR) {
      // Q rows past the tile that phase 1 did not consume at this step (their
      // records come from the step before): phase 2 reads them normalised.
      if (lc || !(stride != 1 || step == 0))
        norm_rope_smem_rows<TE, P>(qslot(step & 1) + T * P, QDR - T, j0 + T, grp, l, nr_weights(p.nq.w, l), p.nq,
                                   p.L);
    }
    __syncthreads();
    // Phase 2 reads no K/V: the next step's K/V copies go out now.
    if constexpr (TMA) {
      if (tid == 0 && step + 1 < n_steps) issue_kv(step + 1);
    } else {
      __syncthreads();
    }

    // ---- Phase 2: dK / dV of own keys, gathered from their consumers. ----
    {
      const int a = grp * 4;
      // Local carry: keys a - d .. a - d + 3 (mod T); "carried" groups hold the
      // last d keys, whose far consumers a .. a + 3 lie in the previous step's tile.
      const bool carried = lc && a < d;
      const int r0 = lc ? (carried ? a - d + T : a - d) : a;
      // Records r0 + j (j = 0..5, fixed after unrolling) and the group's own rows a + i.
      const float* Ea = egroup(r0);
      const float* Eb = egroup(r0 + 4);
      const float* Eo = egroup(a);
      auto rec = [&](int j, int src) {
        return *reinterpret_cast<const float2*>((j < 4 ? Ea + 8 * j : Eb + 8 * (j - 4)) + 2 * src);
      };
      // NR: the group's four raw k rows, all loaded before this phase's first dK/dV
      // store.  A load placed after a store it may alias (as far as the compiler
      // knows) cannot move above it, so loads issued per key each wait out their
      // own round trip to L2.
      RowWords<TE> kraw[4];
      if constexpr (NR && !is_pre) {
        const TE* kb = reinterpret_cast<const TE*>(p.k.ptr) + (long long)b * p.k.sb + (long long)hk * p.k.sh;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = j0 + r0 + i;
          kraw[i] = load_row_words<TE>(kb + (long long)min(j, p.L - 1) * p.k.sl, p.D, l, j < p.L);
        }
      }
      Frag q1 = FragIO<TE>::load(Qs + (r0 + 1) * P, l), d1 = FragIO<TE>::load(Ds + (r0 + 1) * P, l);
      Frag q0 = FragIO<TE>::load(Qs + r0 * P, l), d0 = FragIO<TE>::load(Ds + r0 * P, l);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = r0 + i;
        const Frag q2 = FragIO<TE>::load(Qs + (r + 2) * P, l);
        const Frag d2 = FragIO<TE>::load(Ds + (r + 2) * P, l);
        Frag qf, df;  // local carry: the group's own consumer row a + i
        if (lc) {
          qf = FragIO<TE>::load(Qs + (a + i) * P, l);
          df = FragIO<TE>::load(Ds + (a + i) * P, l);
        }
        if (!is_pre) {
          Frag ak = carry_k[i], av = carry_v[i];
          if (has0) {
            const float2 e = rec(i, 0);
            frag_axpy(ak, e.y, q0);
            frag_axpy(av, e.x, d0);
          }
          if (has1) {
            const float2 e = rec(i + 1, 1);
            frag_axpy(ak, e.y, q1);
            frag_axpy(av, e.x, d1);
          }
          if (has2) {
            const float2 e = rec(i + 2, 2);
            frag_axpy(ak, e.y, q2);
            frag_axpy(av, e.x, d2);
          }
          if (lc && !carried) {
            const float2 e = *reinterpret_cast<const float2*>(Eo + 8 * i + 6);
            frag_axpy(ak, e.y, qf);
            frag_axpy(av, e.x, df);
          } else if (far && !chain && !lc) {
            const int c = r + d;
            const float2 e = *reinterpret_cast<const float2*>(erec(c) + 6);
            frag_axpy(ak, e.y, FragIO<TE>::load(Qs + c * P, l));
            frag_axpy(av, e.x, FragIO<TE>::load(Ds + c * P, l));
          }
          const int j = j0 + r;
          if constexpr (NR) {
            // dK of the raw row: RoPE transpose and RMSNorm Jacobian on the raw k,
            // re-read from global memory (the slot holding it is being refilled).
            const Frag kx = FragIO<TE>::from_words(kraw[i].w);
            const float rk = nr_rsqrt(fmaf(nr_row_dot(kx, kx), 1.f / 64.f, p.nk.eps));
            ak = norm_rope_grad<TE>(ak, kx, rk, l, nr_weights(p.nk.w, l), p.nk, j, p.L, dwk, j < p.L);
          }
          if (j < p.L) {
            store_frag<TO, TMA>(dk + (long long)j * p.dk.sl, p.dk.sd, p.D, l, ak);
            store_frag<TO, TMA>(dv + (long long)j * p.dv.sl, p.dv.sd, p.D, l, av);
          }
        }
        if (chain && far) {
          const float2 e = rec(i, 3);
          carry_k[i] = frag_mul(e.y, q0);
          carry_v[i] = frag_mul(e.x, d0);
        }
        if (carried) {
          const float2 e = *reinterpret_cast<const float2*>(Eo + 8 * i + 6);
          carry_k[i] = frag_mul(e.y, qf);
          carry_v[i] = frag_mul(e.x, df);
        }
        q0 = q1;
        d0 = d1;
        q1 = q2;
        d1 = d2;
      }
    }
    __syncthreads();  // slots of this step are refilled by later copies
    return true;
  };

  auto stop = [&] {  // a copy wait expired: no weight-gradient partial from this CTA
    if constexpr (NR) p.dw_partial[(long long)blockIdx.x * 128 + tid] = 0.f;
  };
  int first = 0;
  if (pre) {
    if (!run_step(0, std::true_type{})) return stop();
    first = 1;
  }
#pragma unroll 1
  for (int step = first; step < n_steps; ++step)
    if (!run_step(step, std::false_type{})) return stop();
  if constexpr (NR) nr_write_partials(p.dw_partial, reinterpret_cast<float*>(QDbase), dwq, dwk, grp, l);
}

// Source-set shapes of a plan: the forward's (sbda_fwd_v2_kernel SHAPE) and the
// backward's (BwdShape); 0 when no specialisation applies.
inline int fwd_shape(const V2Geometry& g, int tile) {
  if (g.has0 && g.has1 && !g.has2 && !g.has_far) return 1;
  if (g.has0 && !g.has1 && g.has2 && !g.has_far) return 2;
  if (g.has0 && g.has1 && g.has2 && g.has_far) return g.d < tile ? 4 : 3;
  return 0;
}

inline int bwd_shape(const V2Geometry& g) {
  if (g.has0 && g.has1 && !g.has2 && !g.has_far) return 1;
  if (g.has0 && !g.has1 && g.has2 && !g.has_far) return 2;
  if (g.has0 && g.has1 && g.has2 && g.has_far) return g.mode == 0 ? 4 : (g.mode == 2 ? 3 : 5);
  return 0;
}

}  // namespace sbda
