// sbda_norm_rope.cu -- per-head RMSNorm + half-split RoPE for the SBDA q/k
// projections, forward and backward, replacing the ~10 eager ops per tensor
// of BiAttn/attention_common.py:13-76 (called at BiAttn/left_v2.py:237-239).
//
// Forward (per row = one head of one position, D channels, h = D / 2):
//   r   = rsqrt(mean_j x_j^2 + eps)                         fp32 (attention_common.py:73-75)
//   y_j = cast(x_j * r * w_j)                               cast to the input dtype (:76)
//   z_j = cast(cast(y_j * c_j) + cast(rot(y)_j * s_j))      RoPE in the input dtype (:48-49)
//   rot(y)_j = -y_{j+h} (j < h),  y_{j-h} (j >= h);  c, s = the position's cos/sin table row
//   (fp32 angles cast to the input dtype, :13-22).  Odd D: z = y (:36-40).
// Backward (fp32, the same function's exact derivative):
//   g_j  = dz_j c_j + (j < h ? dz_{j+h} s_{j+h} : -dz_{j-h} s_{j-h})
//   dx_k = r u_k - x_k r^3 (sum_j u_j x_j) / D,   u = g * w
//   dw_j = sum over every row of g_j x_j r  -- per-CTA partial sums in a workspace
//          and a fixed-order reduction: deterministic, no atomics.
//
// One thread owns one row.  A CTA stages 128 rows in shared memory with a
// row pitch of D*e + 4 bytes (an odd number of words for even D), so the
// lanes of a warp, reading the same channel of 32 consecutive rows, hit
// distinct banks.  Staging loads/stores are warp-per-row and coalesced.
// The backward is a fixed-size grid (at most 2048 / 1024 CTAs, independent
// of the device) walking row blocks; each CTA keeps its weight-gradient
// column sums and writes them once, so the final reduction is short and
// its order is fixed.

#include "sbda_v2_kernels.cuh"  // norm_rope_frag / norm_rope_grad (head_dim 64, 8 lanes per row)

#include <atomic>

namespace sbda {

constexpr int kNRRows = 128;      // rows per CTA step (one per thread)
constexpr int kNRMaxCtas = 1024;  // backward grid cap for head_dim > 64 (twice this at <= 64)

struct NormRopeParams {
  int B, L, H, D;
  int rope;                 // 1 = apply RoPE (even D)
  float eps;
  TensorArg x;              // input rows [B, H, L, D]
  TensorArg y;              // output rows (forward) / grad_x (backward)
  TensorArg dy;             // backward: gradient of the rotated output
  const float* w;           // [D] fp32 weight
  const void* cos_t;        // [table rows, D/2] in the input dtype
  const void* sin_t;
  long long table_offset;   // table row of position 0
  float* partial;           // backward: [gridDim.x, D] fp32 weight-gradient partials
  unsigned* status;         // fault word (bounded copy waits of the ring kernels)
};

template <typename TE>
__device__ __forceinline__ float round_to(float x) {
  return Elem<TE>::to_float(Elem<TE>::from_float(x));
}

// Row index -> (b, position, head); rows are ordered (b, position, head) so
// that the heads of a position are neighbours (contiguous in [B, L, H, D]).
__device__ __forceinline__ void row_coords(long long row, int L, int H, int& b, int& pos, int& h) {
  h = (int)(row % H);
  const long long bl = row / H;
  pos = (int)(bl % L);
  b = (int)(bl / L);
}

// Cooperative staging of a block of rows (warp per row, lanes over channels).
template <typename TE>
__device__ void stage_rows(TE* sm, int pitch, const TensorArg& t, long long row0, long long rows_total, int L,
                           int H, int D) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const TE* src = reinterpret_cast<const TE*>(t.ptr);
  for (int r = warp; r < kNRRows; r += nw) {
    const long long row = row0 + r;
    TE* dst = sm + r * pitch;
    if (row < rows_total) {
      int b, pos, h;
      row_coords(row, L, H, b, pos, h);
      const TE* s = src + (long long)b * t.sb + (long long)h * t.sh + (long long)pos * t.sl;
      for (int c = lane; c < D; c += 32) dst[c] = s[(long long)c * t.sd];
    } else {
      for (int c = lane; c < D; c += 32) dst[c] = Elem<TE>::from_float(0.f);
    }
  }
}

template <typename TE>
__device__ void unstage_rows(const TE* sm, int pitch, const TensorArg& t, long long row0, long long rows_total,
                             int L, int H, int D) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  TE* dst0 = reinterpret_cast<TE*>(const_cast<void*>(t.ptr));
  for (int r = warp; r < kNRRows; r += nw) {
    const long long row = row0 + r;
    if (row >= rows_total) break;
    int b, pos, h;
    row_coords(row, L, H, b, pos, h);
    TE* d = dst0 + (long long)b * t.sb + (long long)h * t.sh + (long long)pos * t.sl;
    const TE* s = sm + r * pitch;
    for (int c = lane; c < D; c += 32) d[(long long)c * t.sd] = s[c];
  }
}

template <typename TE>
__global__ void __launch_bounds__(kNRRows) sbda_norm_rope_fwd_kernel(const NormRopeParams p) {
  extern __shared__ __align__(16) uint8_t nr_smem[];
  TE* sm = reinterpret_cast<TE*>(nr_smem);
  const int D = p.D, pitch = D + 4 / (int)sizeof(TE), half = D / 2;
  const long long rows_total = (long long)p.B * p.L * p.H;
  const long long row0 = (long long)blockIdx.x * kNRRows;
  stage_rows<TE>(sm, pitch, p.x, row0, rows_total, p.L, p.H, D);
  __syncthreads();
  const long long row = row0 + threadIdx.x;
  if (row < rows_total) {
    TE* xr = sm + threadIdx.x * pitch;
    float ss = 0.f;
    for (int j = 0; j < D; ++j) {
      const float v = Elem<TE>::to_float(xr[j]);
      ss = fmaf(v, v, ss);
    }
    const float r = rsqrtf(ss / (float)D + p.eps);
    // y = cast(x * r * w), kept in place
    for (int j = 0; j < D; ++j) xr[j] = Elem<TE>::from_float(Elem<TE>::to_float(xr[j]) * r * p.w[j]);
    if (p.rope) {
      int b, pos, h;
      row_coords(row, p.L, p.H, b, pos, h);
      const TE* ct = reinterpret_cast<const TE*>(p.cos_t) + (p.table_offset + pos) * half;
      const TE* st = reinterpret_cast<const TE*>(p.sin_t) + (p.table_offset + pos) * half;
      for (int j = 0; j < half; ++j) {
        const float c = Elem<TE>::to_float(ct[j]), s = Elem<TE>::to_float(st[j]);
        const float lo = Elem<TE>::to_float(xr[j]), hi = Elem<TE>::to_float(xr[j + half]);
        // z_j = cast(cast(lo*c) + cast(-hi*s)); z_{j+h} = cast(cast(hi*c) + cast(lo*s))
        const float zl = round_to<TE>(round_to<TE>(lo * c) + round_to<TE>(-hi * s));
        const float zh = round_to<TE>(round_to<TE>(hi * c) + round_to<TE>(lo * s));
        xr[j] = Elem<TE>::from_float(zl);
        xr[j + half] = Elem<TE>::from_float(zh);
      }
    }
  }
  __syncthreads();
  unstage_rows<TE>(sm, pitch, p.y, row0, rows_total, p.L, p.H, D);
}

template <typename TE>
__global__ void __launch_bounds__(kNRRows) sbda_norm_rope_bwd_kernel(const NormRopeParams p) {
  extern __shared__ __align__(16) uint8_t nr_smem[];
  const int D = p.D, pitch = D + 4 / (int)sizeof(TE), half = D / 2;
  TE* sx = reinterpret_cast<TE*>(nr_smem);
  TE* sg = sx + kNRRows * pitch;
  float* contrib = reinterpret_cast<float*>(sg + kNRRows * pitch);  // [kNRRows][D + 1]
  const int cpitch = D + 1;
  const long long rows_total = (long long)p.B * p.L * p.H;
  const long long nblocks = (rows_total + kNRRows - 1) / kNRRows;
  float* cr = contrib + threadIdx.x * cpitch;
  for (int j = 0; j < D; ++j) cr[j] = 0.f;
  for (long long blk = blockIdx.x; blk < nblocks; blk += gridDim.x) {
    const long long row0 = blk * kNRRows;
    __syncthreads();  // staging buffers of the previous block are drained
    stage_rows<TE>(sx, pitch, p.x, row0, rows_total, p.L, p.H, D);
    stage_rows<TE>(sg, pitch, p.dy, row0, rows_total, p.L, p.H, D);
    __syncthreads();
    const long long row = row0 + threadIdx.x;
    if (row < rows_total) {
      TE* xr = sx + threadIdx.x * pitch;
      TE* gr = sg + threadIdx.x * pitch;
      float ss = 0.f;
      for (int j = 0; j < D; ++j) {
        const float v = Elem<TE>::to_float(xr[j]);
        ss = fmaf(v, v, ss);
      }
      const float r = rsqrtf(ss / (float)D + p.eps);
      // Two passes over the row: g = RoPE-transposed gradient (recomputed in
      // the second pass rather than stored), dot = sum(g * w * x), then dx.
      float dot = 0.f;
      if (p.rope) {
        int b, pos, h;
        row_coords(row, p.L, p.H, b, pos, h);
        const TE* ct = reinterpret_cast<const TE*>(p.cos_t) + (p.table_offset + pos) * half;
        const TE* st = reinterpret_cast<const TE*>(p.sin_t) + (p.table_offset + pos) * half;
        for (int j = 0; j < half; ++j) {
          const float c = Elem<TE>::to_float(ct[j]), s = Elem<TE>::to_float(st[j]);
          const float dl = Elem<TE>::to_float(gr[j]), dh = Elem<TE>::to_float(gr[j + half]);
          const float gl = dl * c + dh * s, gh = dh * c - dl * s;
          const float xl = Elem<TE>::to_float(xr[j]), xh = Elem<TE>::to_float(xr[j + half]);
          dot = fmaf(gl * p.w[j], xl, dot);
          dot = fmaf(gh * p.w[j + half], xh, dot);
          cr[j] = fmaf(gl * xl, r, cr[j]);
          cr[j + half] = fmaf(gh * xh, r, cr[j + half]);
        }
        const float k3 = r * r * r * dot / (float)D;
        for (int j = 0; j < half; ++j) {
          const float c = Elem<TE>::to_float(ct[j]), s = Elem<TE>::to_float(st[j]);
          const float dl = Elem<TE>::to_float(gr[j]), dh = Elem<TE>::to_float(gr[j + half]);
          const float gl = dl * c + dh * s, gh = dh * c - dl * s;
          const float xl = Elem<TE>::to_float(xr[j]), xh = Elem<TE>::to_float(xr[j + half]);
          gr[j] = Elem<TE>::from_float(r * gl * p.w[j] - xl * k3);
          gr[j + half] = Elem<TE>::from_float(r * gh * p.w[j + half] - xh * k3);
        }
      } else {
        for (int j = 0; j < D; ++j) {
          const float g = Elem<TE>::to_float(gr[j]), x = Elem<TE>::to_float(xr[j]);
          dot = fmaf(g * p.w[j], x, dot);
          cr[j] = fmaf(g * x, r, cr[j]);
        }
        const float k3 = r * r * r * dot / (float)D;
        for (int j = 0; j < D; ++j) {
          const float g = Elem<TE>::to_float(gr[j]), x = Elem<TE>::to_float(xr[j]);
          gr[j] = Elem<TE>::from_float(r * g * p.w[j] - x * k3);
        }
      }
    }
    __syncthreads();
    unstage_rows<TE>(sg, pitch, p.y, row0, rows_total, p.L, p.H, D);
  }
  __syncthreads();
  // Fixed-order column sums of this CTA's rows -> partial[blockIdx.x][j].
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float acc = 0.f;
    for (int rr = 0; rr < kNRRows; ++rr) acc += contrib[rr * cpitch + j];
    p.partial[(long long)blockIdx.x * D + j] = acc;
  }
}

// dw[j] = sum over blocks of partial[block][j] in a fixed order: thread (j, s)
// sums slice s of blockDim.y consecutive row ranges in row order, then the
// slice sums are added in slice order.  The slice count depends on D only, so
// the order is independent of timing and device: deterministic.
constexpr int kDwMaxSlices = 16;

__global__ void __launch_bounds__(1024) sbda_norm_weight_reduce_kernel(const float* __restrict__ partial,
                                                                       int blocks, int D, float* __restrict__ dw) {
  __shared__ float slice_sum[kDwMaxSlices][128];
  const int j = threadIdx.x, sl = threadIdx.y, slices = blockDim.y;
  const int per = (blocks + slices - 1) / slices;
  const int lo = sl * per, hi = min(blocks, lo + per);
  float acc = 0.f;
#pragma unroll 8
  for (int b = lo; b < hi; ++b) acc += partial[(long long)b * D + j];
  slice_sum[sl][j] = acc;
  __syncthreads();
  if (sl == 0) {
    float total = 0.f;
    for (int t = 0; t < slices; ++t) total += slice_sum[t][j];
    dw[j] = total;
  }
}

// --------------------------------------------------------------------------
// head_dim 64 with layouts the vector path takes (16-byte aligned rows and
// strides, unit channel stride, 16-byte aligned tables and weight): 8 lanes
// per row, each lane holding 8 channels in registers, the rotation partner
// one shuffle away (lane ^ 4).  A CTA iteration covers 16 * R rows (R rows
// per lane: kNRFwdRows, kNRBwdRows): row group g takes rows base + 16 i + g
// (i < R), so each warp reads 4 consecutive rows (512 contiguous bytes in the
// [B, L, H, D] layout) per load, and a lane has R rows' loads in flight before
// it computes.
// --------------------------------------------------------------------------

constexpr int kNRFwdRows = 4;  // forward: rows per lane per CTA iteration (16 row groups per CTA)

// n / d for 0 <= n < 2^31 by a multiply and a shift: division by an invariant
// integer with a rounded-up multiplier (Granlund and Montgomery, "Division by
// invariant integers using multiplication", PLDI 1994, theorem 4.2): with
// l = ceil(log2 d) and m = ceil(2^(31 + l) / d) < 2^32, n / d = (n * m) >> (31 + l).
struct FastDiv {
  unsigned d, m, shift;
};

FastDiv make_fastdiv(unsigned d) {
  unsigned l = 0;
  while ((1ull << l) < d) ++l;
  const unsigned long long num = 1ull << (31 + l);
  return FastDiv{d, (unsigned)((num + d - 1) / d), 31 + l};
}

__device__ __forceinline__ unsigned fdiv(unsigned n, const FastDiv& f) {
  return (unsigned)(((unsigned long long)n * f.m) >> f.shift);
}

// Row r of the (batch, position, head) order -> element offset in t and position.
__device__ __forceinline__ void nr_coords(unsigned row, const FastDiv& fh, const FastDiv& fl, int* b, int* pos,
                                          int* h) {
  const unsigned bl = fdiv(row, fh);
  *h = (int)(row - bl * fh.d);
  const unsigned bb = fdiv(bl, fl);
  *pos = (int)(bl - bb * fl.d);
  *b = (int)bb;
}

__device__ __forceinline__ long long nr_offset(const TensorArg& t, int b, int pos, int h) {
  return (long long)b * t.sb + (long long)h * t.sh + (long long)pos * t.sl;
}

template <typename TE>
__global__ void __launch_bounds__(128) sbda_norm_rope64_fwd_kernel(const NormRopeParams p, const FastDiv fh,
                                                                   const FastDiv fl) {
  const int l = threadIdx.x & 7, grp = threadIdx.x >> 3;
  const long long rows_total = (long long)p.B * p.L * p.H;
  const NormRopeArgs a{p.w, p.cos_t, p.sin_t, p.table_offset, p.eps};
  const Frag w = nr_weights(p.w, l);
  const TE* x = reinterpret_cast<const TE*>(p.x.ptr);
  TE* y = reinterpret_cast<TE*>(const_cast<void*>(p.y.ptr));
  for (long long base = (long long)blockIdx.x * 16 * kNRFwdRows; base < rows_total;
       base += (long long)gridDim.x * 16 * kNRFwdRows) {
    RowWords<TE> in[kNRFwdRows];
    RopeWords<TE> rw[kNRFwdRows];
    int pos[kNRFwdRows];
    long long yo[kNRFwdRows];
#pragma unroll
    for (int i = 0; i < kNRFwdRows; ++i) {
      const long long row = base + 16 * i + grp;
      const bool live = row < rows_total;
      int b, h;
      nr_coords((unsigned)(live ? row : rows_total - 1), fh, fl, &b, &pos[i], &h);
      yo[i] = nr_offset(p.y, b, pos[i], h);
      in[i] = load_row_words<TE>(x + nr_offset(p.x, b, pos[i], h), 64, l, live);
      rw[i] = rope_words<TE>(a, pos[i], p.L, l);
    }
#pragma unroll
    for (int i = 0; i < kNRFwdRows; ++i) {
      const Frag z = norm_rope_frag_w<TE>(FragIO<TE>::from_words(in[i].w), l, w, a.eps, rw[i], nullptr);
      if (base + 16 * i + grp < rows_total) store_frag<TE, true>(y + yo[i], 1, 64, l, z);
    }
  }
}

// Rows per lane per iteration of the backward (16 * kNRBwdRows rows per CTA iteration).
constexpr int kNRBwdRows = 2;

// One CTA iteration's input rows of the backward: x and dy of kNRBwdRows rows per lane.
template <typename TE>
struct NR64BwdRows {
  RowWords<TE> x[kNRBwdRows], g[kNRBwdRows];
  RopeWords<TE> rw[kNRBwdRows];
  int pos[kNRBwdRows];
  long long dxo[kNRBwdRows];
};

template <typename TE>
__device__ __forceinline__ void nr64_bwd_load(NR64BwdRows<TE>& r, const NormRopeParams& p, long long base,
                                              long long rows_total, int grp, int l, const FastDiv& fh,
                                              const FastDiv& fl) {
  const TE* x = reinterpret_cast<const TE*>(p.x.ptr);
  const TE* dy = reinterpret_cast<const TE*>(p.dy.ptr);
#pragma unroll
  for (int i = 0; i < kNRBwdRows; ++i) {
    const long long row = base + 16 * i + grp;
    const bool live = row < rows_total;
    int b, h;
    nr_coords((unsigned)(live ? row : rows_total - 1), fh, fl, &b, &r.pos[i], &h);
    r.dxo[i] = nr_offset(p.y, b, r.pos[i], h);
    r.x[i] = load_row_words<TE>(x + nr_offset(p.x, b, r.pos[i], h), 64, l, live);
    r.g[i] = load_row_words<TE>(dy + nr_offset(p.dy, b, r.pos[i], h), 64, l, live);
    r.rw[i] = rope_words<TE>(NormRopeArgs{p.w, p.cos_t, p.sin_t, p.table_offset, p.eps}, r.pos[i], p.L, l);
  }
}

// Loads of an iteration are issued together (2 per row per lane), then its math runs.
// (Loading the next iteration's rows during this one's math needs ~160
// registers: 3 CTAs per SM instead of 4, and measured 22 % slower.)
template <typename TE>
__global__ void __launch_bounds__(128) sbda_norm_rope64_bwd_kernel(const NormRopeParams p, const FastDiv fh,
                                                                   const FastDiv fl) {
  __shared__ float sums[16 * 64];
  const int l = threadIdx.x & 7, grp = threadIdx.x >> 3;
  const long long rows_total = (long long)p.B * p.L * p.H;
  const long long stride = (long long)gridDim.x * 16 * kNRBwdRows;
  const NormRopeArgs a{p.w, p.cos_t, p.sin_t, p.table_offset, p.eps};
  const Frag w = nr_weights(p.w, l);
  TE* dx = reinterpret_cast<TE*>(const_cast<void*>(p.y.ptr));
  Frag dw = frag_zero();
  for (long long base = (long long)blockIdx.x * 16 * kNRBwdRows; base < rows_total; base += stride) {
    NR64BwdRows<TE> cur;
    nr64_bwd_load(cur, p, base, rows_total, grp, l, fh, fl);
#pragma unroll
    for (int i = 0; i < kNRBwdRows; ++i) {
      const bool live = base + 16 * i + grp < rows_total;
      const Frag xv = FragIO<TE>::from_words(cur.x[i].w);
      const float r = nr_rsqrt(fmaf(nr_row_dot(xv, xv), 1.f / 64.f, p.eps));
      const Frag g = norm_rope_grad_w<TE>(FragIO<TE>::from_words(cur.g[i].w), xv, r, l, w, cur.rw[i], dw, live);
      if (live) store_frag<TE, true>(dx + cur.dxo[i], 1, 64, l, g);
    }
  }
  // Fixed-order column sums of this CTA's row groups -> partial[blockIdx.x][j].
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sums[grp * 64 + 8 * l + 2 * i] = dw.v[i].x;
    sums[grp * 64 + 8 * l + 2 * i + 1] = dw.v[i].y;
  }
  __syncthreads();
  if (threadIdx.x < 64) {
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < 16; ++g) acc += sums[g * 64 + threadIdx.x];
    p.partial[(long long)blockIdx.x * 64 + threadIdx.x] = acc;
  }
}

// --------------------------------------------------------------------------
// head_dim 64 on contiguous [B, L, H, D] rows (consecutive in (batch,
// position, head) order, the layout of a projection's output): the register
// kernels' rows, lanes and math, but each CTA walks its chunks of the grid-
// stride order with the next kNRRingStages - 1 chunks already on their way into
// a small ring of shared-memory stages (untiled bulk copies counted on one
// mbarrier per stage), so its loads overlap its math without holding
// registers.  Outputs are bit-identical to the register kernels'; the
// backward's weight-gradient partials are per CTA over the same rows.
// --------------------------------------------------------------------------

// Chosen by A/B runs at config 4 (per launch, bf16): 2 stages of 64-row (forward)
// and 32-row (backward) chunks.  3 and 4 stages, or 128-row forward / 64-row
// backward chunks, leave fewer CTAs per SM and ran slower.
constexpr int kNRRingStages = 2;
constexpr int kNRRingFwdRows = 4;  // rows per lane per chunk
constexpr int kNRRingBwdRows = 2;

template <typename TE, int ROWS, int TENSORS>
struct NRRing {
  static constexpr int kRow = 64 * (int)sizeof(TE);  // bytes per row
  static constexpr int kChunk = ROWS * kRow;          // bytes per chunk and tensor
  static constexpr size_t kSums = TENSORS == 2 ? 16 * 64 * 4 : 0;  // backward: weight-gradient column sums
  static constexpr size_t kSmem = (size_t)kNRRingStages * TENSORS * kChunk + kSums + kNRRingStages * 8;
};

// After an expired copy wait: record it and wait (bounded) for the copies still
// in flight into this CTA's stages (chunks k0 .. k1 - 1), so none lands after exit.
__device__ __forceinline__ void ring_drain(unsigned* status, uint64_t* bars, long long k0, long long k1) {
  if (threadIdx.x == 0 && status) atomicOr(status, kFaultWaitExpired);
  for (long long k = k0; k < k1; ++k)
    (void)mbar_wait_bounded(bars + k % kNRRingStages, (uint32_t)((k / kNRRingStages) & 1));
}

// x (and dy) of ring chunk k of this CTA: rows [(blockIdx.x + k * gridDim.x) * ROWS, ...).
template <typename TE, int ROWS, int TENSORS>
__device__ __forceinline__ void ring_issue(uint8_t* ring, uint64_t* bars, const void* x, const void* dy, long long k,
                                          long long rows_total) {
  using R = NRRing<TE, ROWS, TENSORS>;
  const long long r0 = ((long long)blockIdx.x + k * gridDim.x) * ROWS;
  const uint32_t bytes = (uint32_t)(min((long long)ROWS, rows_total - r0) * R::kRow);
  uint64_t* bar = bars + k % kNRRingStages;
  uint8_t* dst = ring + (k % kNRRingStages) * TENSORS * R::kChunk;
  mbar_arrive_expect_tx(bar, TENSORS * bytes);
  bulk_load(dst, static_cast<const uint8_t*>(x) + r0 * R::kRow, bytes, bar);
  if (TENSORS == 2) bulk_load(dst + R::kChunk, static_cast<const uint8_t*>(dy) + r0 * R::kRow, bytes, bar);
}

template <typename TE>
__global__ void __launch_bounds__(128) sbda_norm_rope64_fwd_ring_kernel(const NormRopeParams p, const FastDiv fh,
                                                                        const FastDiv fl) {
  constexpr int ROWS = 16 * kNRRingFwdRows;
  using R = NRRing<TE, ROWS, 1>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kNRRingStages * R::kChunk);
  const int tid = threadIdx.x, l = tid & 7, grp = tid >> 3;
  const long long rows_total = (long long)p.B * p.L * p.H;
  const long long chunks = (rows_total + ROWS - 1) / ROWS;
  const long long n = blockIdx.x < chunks ? (chunks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (tid == 0) {
    for (int s = 0; s < kNRRingStages; ++s) mbar_init(bars + s, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0)
    for (long long k = 0; k < n && k < kNRRingStages; ++k) ring_issue<TE, ROWS, 1>(smem, bars, p.x.ptr, nullptr, k, rows_total);
  const NormRopeArgs a{p.w, p.cos_t, p.sin_t, p.table_offset, p.eps};
  const Frag w = nr_weights(p.w, l);
  TE* y = reinterpret_cast<TE*>(const_cast<void*>(p.y.ptr));
  for (long long k = 0; k < n; ++k) {
    // The chunk's coordinates and table words first: they overlap the stage's wait.
    const long long r0 = ((long long)blockIdx.x + k * gridDim.x) * ROWS;
    int pos[kNRRingFwdRows];
    long long yo[kNRRingFwdRows];
    RopeWords<TE> rw[kNRRingFwdRows];
#pragma unroll
    for (int i = 0; i < kNRRingFwdRows; ++i) {
      const long long row = r0 + 16 * i + grp;
      int b, h;
      nr_coords((unsigned)(row < rows_total ? row : rows_total - 1), fh, fl, &b, &pos[i], &h);
      yo[i] = nr_offset(p.y, b, pos[i], h);
      rw[i] = rope_words<TE>(a, pos[i], p.L, l);
    }
    const bool ok = mbar_wait_bounded(bars + k % kNRRingStages, (uint32_t)((k / kNRRingStages) & 1));
    if (__syncthreads_or(!ok)) {
      ring_drain(p.status, bars, k, min(n, k + kNRRingStages));
      return;
    }
    const uint8_t* st = smem + (k % kNRRingStages) * R::kChunk;
#pragma unroll
    for (int i = 0; i < kNRRingFwdRows; ++i) {
      // Rows past the tensor's end compute on stale stage bytes and store nothing.
      const int rr = 16 * i + grp;
      const Frag z = norm_rope_frag_w<TE>(FragIO<TE>::load(st + rr * R::kRow, l), l, w, a.eps, rw[i], nullptr);
      if (r0 + rr < rows_total) store_frag<TE, true>(y + yo[i], 1, 64, l, z);
    }
    __syncthreads();  // every thread is done with this stage
    if (tid == 0 && k + kNRRingStages < n)
      ring_issue<TE, ROWS, 1>(smem, bars, p.x.ptr, nullptr, k + kNRRingStages, rows_total);
  }
}

// Backward: the register kernel's grid, with the same rows per CTA (chunks c,
// c + grid, ...) and the same per-CTA partial rows, bit for bit.
template <typename TE>
__global__ void __launch_bounds__(128) sbda_norm_rope64_bwd_ring_kernel(const NormRopeParams p, const FastDiv fh,
                                                                        const FastDiv fl) {
  constexpr int ROWS = 16 * kNRRingBwdRows;
  using R = NRRing<TE, ROWS, 2>;
  extern __shared__ __align__(128) uint8_t smem[];
  float* sums = reinterpret_cast<float*>(smem + kNRRingStages * 2 * R::kChunk);  // [16 row groups][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sums + 16 * 64);
  const int tid = threadIdx.x, l = tid & 7, grp = tid >> 3;
  const long long rows_total = (long long)p.B * p.L * p.H;
  const long long chunks = (rows_total + ROWS - 1) / ROWS;
  const long long n = blockIdx.x < chunks ? (chunks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (tid == 0) {
    for (int s = 0; s < kNRRingStages; ++s) mbar_init(bars + s, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0)
    for (long long k = 0; k < n && k < kNRRingStages; ++k)
      ring_issue<TE, ROWS, 2>(smem, bars, p.x.ptr, p.dy.ptr, k, rows_total);
  const NormRopeArgs a{p.w, p.cos_t, p.sin_t, p.table_offset, p.eps};
  const Frag w = nr_weights(p.w, l);
  TE* dx = reinterpret_cast<TE*>(const_cast<void*>(p.y.ptr));
  Frag dw = frag_zero();
  for (long long k = 0; k < n; ++k) {
    // The chunk's coordinates and table words first: they overlap the stage's wait.
    const long long r0 = ((long long)blockIdx.x + k * gridDim.x) * ROWS;
    long long dxo[kNRRingBwdRows];
    RopeWords<TE> rw[kNRRingBwdRows];
#pragma unroll
    for (int i = 0; i < kNRRingBwdRows; ++i) {
      const long long row = r0 + 16 * i + grp;
      int b, pos, h;
      nr_coords((unsigned)(row < rows_total ? row : rows_total - 1), fh, fl, &b, &pos, &h);
      dxo[i] = nr_offset(p.y, b, pos, h);
      rw[i] = rope_words<TE>(a, pos, p.L, l);
    }
    const bool ok = mbar_wait_bounded(bars + k % kNRRingStages, (uint32_t)((k / kNRRingStages) & 1));
    if (__syncthreads_or(!ok)) {
      // No partial row from this CTA: the fault word marks the result invalid.
      ring_drain(p.status, bars, k, min(n, k + kNRRingStages));
      return;
    }
    const uint8_t* st = smem + (k % kNRRingStages) * 2 * R::kChunk;
#pragma unroll
    for (int i = 0; i < kNRRingBwdRows; ++i) {
      const int rr = 16 * i + grp;
      const bool live = r0 + rr < rows_total;
      const Frag xv = FragIO<TE>::load(st + rr * R::kRow, l);
      const float r = nr_rsqrt(fmaf(nr_row_dot(xv, xv), 1.f / 64.f, p.eps));
      const Frag g =
          norm_rope_grad_w<TE>(FragIO<TE>::load(st + R::kChunk + rr * R::kRow, l), xv, r, l, w, rw[i], dw, live);
      if (live) store_frag<TE, true>(dx + dxo[i], 1, 64, l, g);
    }
    __syncthreads();  // every thread is done with this stage
    if (tid == 0 && k + kNRRingStages < n)
      ring_issue<TE, ROWS, 2>(smem, bars, p.x.ptr, p.dy.ptr, k + kNRRingStages, rows_total);
  }
  // Fixed-order column sums of this CTA's row groups -> partial[blockIdx.x][j].
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sums[grp * 64 + 8 * l + 2 * i] = dw.v[i].x;
    sums[grp * 64 + 8 * l + 2 * i + 1] = dw.v[i].y;
  }
  __syncthreads();
  if (tid < 64) {
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < 16; ++g) acc += sums[g * 64 + tid];
    p.partial[(long long)blockIdx.x * 64 + tid] = acc;
  }
}

// The vector path's preconditions (host side).
bool nr_vec_ok(const TensorArg& t, int e) {
  if (reinterpret_cast<uintptr_t>(t.ptr) % 16 || t.sd != 1) return false;
  return (t.sb * e) % 16 == 0 && (t.sh * e) % 16 == 0 && (t.sl * e) % 16 == 0;
}

bool nr_use64(const NormRopeParams& p, int e, bool backward) {
  if (p.D != 64 || !p.rope) return false;
  if ((long long)p.B * p.L * p.H >= (1ll << 31)) return false;  // 31-bit row indices (FastDiv)
  if (reinterpret_cast<uintptr_t>(p.w) % 16 || reinterpret_cast<uintptr_t>(p.cos_t) % 16 ||
      reinterpret_cast<uintptr_t>(p.sin_t) % 16)
    return false;
  return nr_vec_ok(p.x, e) && nr_vec_ok(p.y, e) && (!backward || nr_vec_ok(p.dy, e));
}

// Contiguous [B, L, H, D] rows of 64 channels: row r of the (batch, position,
// head) order starts at element 64 r (a size-1 dimension may have any stride).
bool nr_rows_contiguous(const TensorArg& t, const NormRopeParams& p) {
  return t.sd == 1 && (p.H == 1 || t.sh == 64) && (p.L == 1 || t.sl == 64LL * p.H) &&
         (p.B == 1 || t.sb == 64LL * p.H * p.L);
}

template <typename TE>
int nr_forward(const NormRopeParams& p, unsigned blocks, cudaStream_t st) {
  if (nr_use64(p, sizeof(TE), false) && nr_rows_contiguous(p.x, p)) {
    // Every CTA resident at once (SMs x CTAs per SM), each walking several chunks.
    auto kern = sbda_norm_rope64_fwd_ring_kernel<TE>;
    const size_t smem = NRRing<TE, 16 * kNRRingFwdRows, 1>::kSmem;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return SBDA_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 128, smem) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    const long long chunks = ((long long)p.B * p.L * p.H + 16 * kNRRingFwdRows - 1) / (16 * kNRRingFwdRows);
    const long long cap = (long long)sm_count() * per_sm;
    kern<<<(unsigned)(chunks < cap ? chunks : cap), 128, smem, st>>>(p, make_fastdiv((unsigned)p.H),
                                                                    make_fastdiv((unsigned)p.L));
    return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
  }
  if (nr_use64(p, sizeof(TE), false)) {
    const long long rows = (long long)p.B * p.L * p.H;
    const long long grid = (rows + 16 * kNRFwdRows - 1) / (16 * kNRFwdRows);
    sbda_norm_rope64_fwd_kernel<TE><<<(unsigned)(grid < (1ll << 20) ? grid : (1ll << 20)), 128, 0, st>>>(
        p, make_fastdiv((unsigned)p.H), make_fastdiv((unsigned)p.L));
    return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
  }
  const size_t smem = (size_t)kNRRows * (p.D * sizeof(TE) + 4);
  auto kern = sbda_norm_rope_fwd_kernel<TE>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SBDA_ERR_CUDA;
  kern<<<blocks, kNRRows, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE>
int nr_backward(const NormRopeParams& p, unsigned blocks, float* grad_w, cudaStream_t st) {
  if (nr_use64(p, sizeof(TE), true) && nr_rows_contiguous(p.x, p) && nr_rows_contiguous(p.dy, p)) {
    // Same grid and rows per CTA as the register kernel below: the same partials.
    auto kern = sbda_norm_rope64_bwd_ring_kernel<TE>;
    const size_t smem = NRRing<TE, 16 * kNRRingBwdRows, 2>::kSmem;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return SBDA_ERR_CUDA;
    kern<<<blocks, 128, smem, st>>>(p, make_fastdiv((unsigned)p.H), make_fastdiv((unsigned)p.L));
  } else if (nr_use64(p, sizeof(TE), true)) {
    // `blocks` CTAs (a cap that depends on head_dim only, not the device) walk the rows, so
    // the partials and their summation order do not depend on the GPU.
    sbda_norm_rope64_bwd_kernel<TE><<<blocks, 128, 0, st>>>(p, make_fastdiv((unsigned)p.H),
                                                             make_fastdiv((unsigned)p.L));
  } else {
    const size_t smem = (size_t)kNRRows * (2 * (p.D * sizeof(TE) + 4) + (p.D + 1) * sizeof(float));
    auto kern = sbda_norm_rope_bwd_kernel<TE>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return SBDA_ERR_CUDA;
    kern<<<blocks, kNRRows, smem, st>>>(p);
  }
  if (cudaGetLastError() != cudaSuccess) return SBDA_ERR_CUDA;
  const int slices = p.D <= 64 ? kDwMaxSlices : kDwMaxSlices / 2;  // D * slices <= 1024 threads
  sbda_norm_weight_reduce_kernel<<<1, dim3(p.D, slices), 0, st>>>(p.partial, (int)blocks, p.D, grad_w);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

int64_t norm_rope_blocks(const sbda_shape& s) {
  const int64_t rows = s.batch * s.length * s.heads;
  return (rows + kNRRows - 1) / kNRRows;
}

// Backward grid: one CTA per row block up to a cap that depends only on the
// head size (device-independent, so the weight-gradient summation order is
// too): 2 * kNRMaxCtas for head_dim <= 64, kNRMaxCtas above.  Either way the
// partials fit in kNRMaxCtas * 128 floats.
int64_t norm_rope_bwd_ctas(const sbda_shape& s) {
  const int64_t b = norm_rope_blocks(s);
  const int64_t cap = s.head_dim <= 64 ? 2 * kNRMaxCtas : kNRMaxCtas;
  return b < cap ? b : cap;
}

int norm_rope_check(int dtype, const sbda_shape& s, float eps) {
  if (dtype != SBDA_DTYPE_F32 && dtype != SBDA_DTYPE_F16 && dtype != SBDA_DTYPE_BF16) return SBDA_ERR_DTYPE;
  if (s.batch < 0 || s.heads < 0 || s.length < 0 || s.head_dim < 1 || s.head_dim > 128) return SBDA_ERR_INVALID;
  if (!(eps >= 0.f)) return SBDA_ERR_INVALID;
  if (s.length > ((int64_t)1 << 31) - 1 || norm_rope_blocks(s) > ((int64_t)1 << 31) - 1) return SBDA_ERR_UNSUPPORTED;
  return SBDA_OK;
}

NormRopeParams nr_params(const sbda_shape& s, const sbda_tensor& x, const sbda_tensor& y, const float* w,
                         float eps, const void* cos_t, const void* sin_t, int64_t table_offset) {
  NormRopeParams p;
  memset(&p, 0, sizeof(p));
  p.B = (int)s.batch;
  p.L = (int)s.length;
  p.H = (int)s.heads;
  p.D = (int)s.head_dim;
  p.rope = (s.head_dim % 2 == 0) && cos_t && sin_t;
  p.eps = eps;
  p.x = TensorArg{x.data, x.stride_b, x.stride_h, x.stride_l, x.stride_d};
  p.y = TensorArg{y.data, y.stride_b, y.stride_h, y.stride_l, y.stride_d};
  p.w = w;
  p.cos_t = cos_t;
  p.sin_t = sin_t;
  p.table_offset = table_offset;
  p.status = status_ptr();
  return p;
}

}  // namespace sbda

using namespace sbda;

extern "C" int64_t sbda_b200_norm_rope_workspace_floats(sbda_shape shape) {
  if (shape.head_dim < 1 || shape.batch < 0 || shape.heads < 0 || shape.length < 0) return 0;
  return norm_rope_bwd_ctas(shape) * shape.head_dim;
}

extern "C" int sbda_b200_norm_rope_forward(int dtype, sbda_shape shape, sbda_tensor x, sbda_tensor y,
                                           const float* weight, float eps, const void* cos_table,
                                           const void* sin_table, int64_t table_offset, void* stream) {
  int st = norm_rope_check(dtype, shape, eps);
  if (st != SBDA_OK) return st;
  if (shape.batch == 0 || shape.heads == 0 || shape.length == 0) return SBDA_OK;
  if (!x.data || !y.data || !weight) return SBDA_ERR_INVALID;
  if (shape.head_dim % 2 == 0 && (!cos_table || !sin_table)) return SBDA_ERR_INVALID;
  const NormRopeParams p = nr_params(shape, x, y, weight, eps, cos_table, sin_table, table_offset);
  const unsigned blocks = (unsigned)norm_rope_blocks(shape);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == SBDA_DTYPE_F32) return nr_forward<float>(p, blocks, s);
  if (dtype == SBDA_DTYPE_F16) return nr_forward<__half>(p, blocks, s);
  return nr_forward<__nv_bfloat16>(p, blocks, s);
}

extern "C" int sbda_b200_norm_rope_backward(int dtype, sbda_shape shape, sbda_tensor x, sbda_tensor grad_y,
                                            const float* weight, float eps, const void* cos_table,
                                            const void* sin_table, int64_t table_offset, sbda_tensor grad_x,
                                            float* grad_weight, float* workspace, int64_t workspace_floats,
                                            void* stream) {
  int st = norm_rope_check(dtype, shape, eps);
  if (st != SBDA_OK) return st;
  if (!grad_weight) return SBDA_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (shape.batch == 0 || shape.heads == 0 || shape.length == 0) {
    return cudaMemsetAsync(grad_weight, 0, sizeof(float) * shape.head_dim, s) == cudaSuccess ? SBDA_OK
                                                                                             : SBDA_ERR_CUDA;
  }
  if (!x.data || !grad_y.data || !grad_x.data || !weight || !workspace) return SBDA_ERR_INVALID;
  if (shape.head_dim % 2 == 0 && (!cos_table || !sin_table)) return SBDA_ERR_INVALID;
  if (workspace_floats < sbda_b200_norm_rope_workspace_floats(shape)) return SBDA_ERR_INVALID;
  NormRopeParams p = nr_params(shape, x, grad_x, weight, eps, cos_table, sin_table, table_offset);
  p.dy = TensorArg{grad_y.data, grad_y.stride_b, grad_y.stride_h, grad_y.stride_l, grad_y.stride_d};
  p.partial = workspace;
  const unsigned blocks = (unsigned)norm_rope_bwd_ctas(shape);
  if (dtype == SBDA_DTYPE_F32) return nr_backward<float>(p, blocks, grad_weight, s);
  if (dtype == SBDA_DTYPE_F16) return nr_backward<__half>(p, blocks, grad_weight, s);
  return nr_backward<__nv_bfloat16>(p, blocks, grad_weight, s);
}

// --------------------------------------------------------------------------
// Allocation-free backward.
//
// Some callers cannot allocate device memory at the point where they run
// the backward: code replayed inside a captured CUDA graph whose memory pool
// is fixed, custom runtimes that hand out only the tensors they planned, or
// plugin hosts that forbid allocation in the execution callback.  For them
// the weight-gradient partials live in this file-scope array instead of a
// caller workspace.  It holds kNoAllocScratchFloats floats (512 KiB: 1024
// CTAs x 128 channels, or 2048 CTAs x 64 channels at head_dim <= 64; enough for
// every shape the backward accepts) on every
// GPU that loads the library, until the process exits.
//
// Every call shares the array.  Each CTA overwrites its partial row before
// the reduction reads it, so nothing needs clearing between calls, but two
// calls that overlap on the GPU (different streams, or different host
// threads on one device) race on it: serialise them.
// --------------------------------------------------------------------------

namespace sbda {

constexpr int64_t kNoAllocScratchFloats = (int64_t)kNRMaxCtas * 128;

static __device__ __align__(256) float g_norm_rope_scratch[kNoAllocScratchFloats];

// Device address of g_norm_rope_scratch for the current device, resolved
// once per device (the host-side symbol is not a device pointer).
float* norm_rope_scratch_ptr(int* status) {
  static std::atomic<float*> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = SBDA_ERR_CUDA;
    return nullptr;
  }
  float* p = cache[dev].load(std::memory_order_acquire);
  if (p) return p;
  void* addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_norm_rope_scratch) != cudaSuccess || !addr) {
    *status = SBDA_ERR_CUDA;
    return nullptr;
  }
  cache[dev].store(static_cast<float*>(addr), std::memory_order_release);
  return static_cast<float*>(addr);
}

}  // namespace sbda

extern "C" int sbda_b200_norm_rope_backward_noalloc(int dtype, sbda_shape shape, sbda_tensor x,
                                                    sbda_tensor grad_y, const float* weight, float eps,
                                                    const void* cos_table, const void* sin_table,
                                                    int64_t table_offset, sbda_tensor grad_x,
                                                    float* grad_weight, void* stream) {
  int st = norm_rope_check(dtype, shape, eps);
  if (st != SBDA_OK) return st;
  if (!grad_weight) return SBDA_ERR_INVALID;
  const int64_t need = sbda_b200_norm_rope_workspace_floats(shape);
  if (need > kNoAllocScratchFloats) return SBDA_ERR_UNSUPPORTED;  // beyond the static scratch
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (shape.batch == 0 || shape.heads == 0 || shape.length == 0) {
    return cudaMemsetAsync(grad_weight, 0, sizeof(float) * shape.head_dim, s) == cudaSuccess ? SBDA_OK
                                                                                             : SBDA_ERR_CUDA;
  }
  if (!x.data || !grad_y.data || !grad_x.data || !weight) return SBDA_ERR_INVALID;
  if (shape.head_dim % 2 == 0 && (!cos_table || !sin_table)) return SBDA_ERR_INVALID;
  int status = SBDA_OK;
  float* scratch = norm_rope_scratch_ptr(&status);
  if (!scratch) return status;
  NormRopeParams p = nr_params(shape, x, grad_x, weight, eps, cos_table, sin_table, table_offset);
  p.dy = TensorArg{grad_y.data, grad_y.stride_b, grad_y.stride_h, grad_y.stride_l, grad_y.stride_d};
  p.partial = scratch;
  const unsigned blocks = (unsigned)norm_rope_bwd_ctas(shape);
  if (dtype == SBDA_DTYPE_F32) return nr_backward<float>(p, blocks, grad_weight, s);
  if (dtype == SBDA_DTYPE_F16) return nr_backward<__half>(p, blocks, grad_weight, s);
  return nr_backward<__nv_bfloat16>(p, blocks, grad_weight, s);
}
