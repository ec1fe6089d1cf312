// sbda_block.cu -- the elementwise parts of the reference block around the
// attention op (BiAttn/model.py:299-335): residual add, padding-row mask and
// RMSNorm in one pass over the residual stream, and the SwiGLU gate.
//
//   residual + norm:  x1 = cast(x + m * a)          (model.py:325 with the
//                                                      attention's row mask, left_v2.py:404)
//                     r  = rsqrt(mean_j x1_j^2 + eps)  fp32 (model.py:25-29, F.rms_norm)
//                     y  = cast(x1 * r * w)
//   backward (fp32):  u = dy * w,  dx1 = r u - x1 r^3 (sum_j u_j x1_j) / dim + dx1_ext
//                     dx = dx1, da = m * dx1, dw = sum over rows of dy * x1 * r
//   SwiGLU gate:      h = cast(cast(silu(g)) * u)    (model.py:58-59, each op in the
//                                                      input dtype as eager torch runs it)
//
// One warp owns one row of `dim` channels (dim % 8 == 0, at most 2048): lane l
// holds 8-channel chunks l, l + 32, ... in registers, so each tensor is read
// once.  The weight gradient is deterministic: per-CTA column sums over the
// rows a CTA walks (fixed grid) go to a caller workspace, then a fixed-order
// reduction.

#include "sbda_common.cuh"

namespace sbda {

constexpr int kBlkWarps = 8;       // rows per CTA step
constexpr int kBlkMaxCtas = 1024;  // backward grid cap (weight-gradient partials)

template <typename TE>
struct Chunk8 {
  static __device__ __forceinline__ void load(const TE* p, float* f) {
    if constexpr (sizeof(TE) == 4) {
      const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
      f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
    } else {
      Elem<TE>::unpack(*reinterpret_cast<const uint4*>(p), f);
    }
  }
  static __device__ __forceinline__ void store(TE* p, const float* f) {
    if constexpr (sizeof(TE) == 4) {
      *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
      *reinterpret_cast<float4*>(p + 4) = make_float4(f[4], f[5], f[6], f[7]);
    } else {
      *reinterpret_cast<uint4*>(p) = Elem<TE>::pack(f);
    }
  }
};

template <typename TE>
__device__ __forceinline__ float round_te(float x) {
  return Elem<TE>::to_float(Elem<TE>::from_float(x));
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) x += __shfl_xor_sync(0xffffffffu, x, m);
  return x;
}

struct BlockNormParams {
  long long rows;
  int dim;
  float eps;
  const void* x;          // forward input (or x1 in the backward)
  const void* add;        // forward: residual addend a (nullable)
  const uint8_t* mask;    // per-row mask m (nullable = all rows kept)
  const float* w;         // [dim] fp32
  void* x1;               // forward: x + m a (written when add != null)
  void* y;                // forward: normalised output
  float* rstd;            // [rows] (forward writes, backward reads)
  const void* dy;         // backward: gradient of y
  const void* dx1_ext;    // backward: gradient reaching x1 from elsewhere (nullable)
  void* dx;               // backward: gradient of x (= of x1)
  void* dadd;             // backward: gradient of a (nullable)
  float* partial;         // backward: [gridDim.x, dim] weight-gradient column sums
};

template <typename TE, int CH>
__global__ void __launch_bounds__(kBlkWarps * 32) sbda_add_rms_norm_fwd_kernel(const BlockNormParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const TE* x = static_cast<const TE*>(p.x);
  const TE* add = static_cast<const TE*>(p.add);
  TE* x1 = static_cast<TE*>(p.x1);
  TE* y = static_cast<TE*>(p.y);
  for (long long row = (long long)blockIdx.x * kBlkWarps + warp; row < p.rows;
       row += (long long)gridDim.x * kBlkWarps) {
    const long long base = row * p.dim;
    const bool keep = p.mask == nullptr || p.mask[row] != 0;
    float v[CH][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int e0 = (c * 32 + lane) * 8;
      if (e0 < p.dim) {
        Chunk8<TE>::load(x + base + e0, v[c]);
        if (add) {
          float a[8];
          Chunk8<TE>::load(add + base + e0, a);
#pragma unroll
          for (int k = 0; k < 8; ++k) v[c][k] = round_te<TE>(v[c][k] + (keep ? a[k] : 0.f));
          Chunk8<TE>::store(x1 + base + e0, v[c]);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) ss = fmaf(v[c][k], v[c][k], ss);
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)p.dim + p.eps);
    if (lane == 0) p.rstd[row] = r;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int e0 = (c * 32 + lane) * 8;
      if (e0 < p.dim) {
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = v[c][k] * r * p.w[e0 + k];
        Chunk8<TE>::store(y + base + e0, o);
      }
    }
  }
}

template <typename TE, int CH>
__global__ void __launch_bounds__(kBlkWarps * 32) sbda_add_rms_norm_bwd_kernel(const BlockNormParams p) {
  extern __shared__ float part[];  // [kBlkWarps][dim] column sums of each warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const TE* x1 = static_cast<const TE*>(p.x);
  const TE* dy = static_cast<const TE*>(p.dy);
  const TE* ext = static_cast<const TE*>(p.dx1_ext);
  TE* dx = static_cast<TE*>(p.dx);
  TE* dadd = static_cast<TE*>(p.dadd);
  float dw[CH][8];
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int k = 0; k < 8; ++k) dw[c][k] = 0.f;
  for (long long row = (long long)blockIdx.x * kBlkWarps + warp; row < p.rows;
       row += (long long)gridDim.x * kBlkWarps) {
    const long long base = row * p.dim;
    const float r = p.rstd[row];
    float xh[CH][8], u[CH][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int e0 = (c * 32 + lane) * 8;
      if (e0 < p.dim) {
        float g[8];
        Chunk8<TE>::load(x1 + base + e0, xh[c]);
        Chunk8<TE>::load(dy + base + e0, g);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          xh[c][k] *= r;
          u[c][k] = g[k] * p.w[e0 + k];
          dot = fmaf(u[c][k], xh[c][k], dot);
          dw[c][k] = fmaf(g[k], xh[c][k], dw[c][k]);
        }
      }
    }
    dot = warp_sum(dot) / (float)p.dim;
    const bool keep = p.mask == nullptr || p.mask[row] != 0;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int e0 = (c * 32 + lane) * 8;
      if (e0 < p.dim) {
        float o[8], e[8];
        if (ext) Chunk8<TE>::load(ext + base + e0, e);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = r * (u[c][k] - xh[c][k] * dot) + (ext ? e[k] : 0.f);
        Chunk8<TE>::store(dx + base + e0, o);
        if (dadd) {
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] = keep ? o[k] : 0.f;
          Chunk8<TE>::store(dadd + base + e0, o);
        }
      }
    }
  }
  // Column sums of this CTA, warps added in a fixed order.
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int e0 = (c * 32 + lane) * 8;
    if (e0 < p.dim)
#pragma unroll
      for (int k = 0; k < 8; ++k) part[warp * p.dim + e0 + k] = dw[c][k];
  }
  __syncthreads();
  for (int j = threadIdx.x; j < p.dim; j += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < kBlkWarps; ++w) s += part[w * p.dim + j];
    p.partial[(long long)blockIdx.x * p.dim + j] = s;
  }
}

__global__ void sbda_block_weight_reduce_kernel(const float* partial, int ctas, int dim, float* out) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= dim) return;
  float s = 0.f;
  for (int c = 0; c < ctas; ++c) s += partial[(long long)c * dim + j];
  out[j] = s;
}

template <typename TE>
__global__ void sbda_silu_mul_fwd_kernel(long long n8, const TE* g, const TE* u, TE* h) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    float a[8], b[8], o[8];
    Chunk8<TE>::load(g + i * 8, a);
    Chunk8<TE>::load(u + i * 8, b);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float s = round_te<TE>(a[k] / (1.f + expf(-a[k])));
      o[k] = s * b[k];
    }
    Chunk8<TE>::store(h + i * 8, o);
  }
}

// d(silu(g) * u): du = dh * silu(g), dg = (dh * u) * sigmoid(g) * (1 + g * (1 - sigmoid(g))),
// each product rounded to the input dtype as eager autograd does.
template <typename TE>
__global__ void sbda_silu_mul_bwd_kernel(long long n8, const TE* g, const TE* u, const TE* dh, TE* dg, TE* du) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    float a[8], b[8], d[8], og[8], ou[8];
    Chunk8<TE>::load(g + i * 8, a);
    Chunk8<TE>::load(u + i * 8, b);
    Chunk8<TE>::load(dh + i * 8, d);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float sg = 1.f / (1.f + expf(-a[k]));
      const float s = round_te<TE>(a[k] * sg);
      ou[k] = d[k] * s;
      const float ds = round_te<TE>(d[k] * b[k]);
      og[k] = ds * sg * (1.f + a[k] * (1.f - sg));
    }
    Chunk8<TE>::store(dg + i * 8, og);
    Chunk8<TE>::store(du + i * 8, ou);
  }
}

namespace {

int block_ctas(long long rows) {
  const long long need = (rows + kBlkWarps - 1) / kBlkWarps;
  return (int)(need < kBlkMaxCtas ? (need > 0 ? need : 1) : kBlkMaxCtas);
}

template <typename TE>
int launch_norm(bool fwd, const BlockNormParams& p, cudaStream_t st) {
  const int chunks = (p.dim + 255) / 256;
  const long long need = (p.rows + kBlkWarps - 1) / kBlkWarps;
  const int ctas = fwd ? (int)(need < 148LL * 32 ? need : 148LL * 32) : block_ctas(p.rows);
  const size_t smem = fwd ? 0 : (size_t)kBlkWarps * p.dim * sizeof(float);
  if (!fwd && smem > 48 * 1024) {
    cudaError_t e = cudaSuccess;
    if (chunks <= 4) e = cudaFuncSetAttribute(sbda_add_rms_norm_bwd_kernel<TE, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    else e = cudaFuncSetAttribute(sbda_add_rms_norm_bwd_kernel<TE, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return SBDA_ERR_CUDA;
  }
#define SBDA_NORM_CASE(CH)                                                                      \
  case CH:                                                                                      \
    if (fwd)                                                                                    \
      sbda_add_rms_norm_fwd_kernel<TE, CH><<<ctas, kBlkWarps * 32, 0, st>>>(p);                 \
    else                                                                                        \
      sbda_add_rms_norm_bwd_kernel<TE, CH><<<ctas, kBlkWarps * 32, smem, st>>>(p);              \
    break;
  switch (chunks) {
    SBDA_NORM_CASE(1)
    SBDA_NORM_CASE(2)
    SBDA_NORM_CASE(4)
    SBDA_NORM_CASE(8)
    case 3:
      if (fwd) sbda_add_rms_norm_fwd_kernel<TE, 4><<<ctas, kBlkWarps * 32, 0, st>>>(p);
      else sbda_add_rms_norm_bwd_kernel<TE, 4><<<ctas, kBlkWarps * 32, smem, st>>>(p);
      break;
    case 5:
    case 6:
    case 7:
      if (fwd) sbda_add_rms_norm_fwd_kernel<TE, 8><<<ctas, kBlkWarps * 32, 0, st>>>(p);
      else sbda_add_rms_norm_bwd_kernel<TE, 8><<<ctas, kBlkWarps * 32, smem, st>>>(p);
      break;
    default:
      return SBDA_ERR_UNSUPPORTED;
  }
#undef SBDA_NORM_CASE
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

int norm_dispatch(int dtype, bool fwd, const BlockNormParams& p, cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return launch_norm<float>(fwd, p, st);
  if (dtype == SBDA_DTYPE_F16) return launch_norm<__half>(fwd, p, st);
  return launch_norm<__nv_bfloat16>(fwd, p, st);
}

bool block_dims_ok(int dtype, long long rows, long long dim) {
  if (dtype != SBDA_DTYPE_F32 && dtype != SBDA_DTYPE_F16 && dtype != SBDA_DTYPE_BF16) return false;
  return rows >= 0 && dim >= 8 && dim <= 2048 && dim % 8 == 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace sbda

using namespace sbda;

extern "C" int sbda_b200_rms_norm_forward(int dtype, int64_t rows, int64_t dim, const void* x,
                                          const void* residual_add, const uint8_t* row_mask,
                                          const float* weight, float eps, void* x1_out, void* y,
                                          float* rstd, void* stream) {
  if (dtype != SBDA_DTYPE_F32 && dtype != SBDA_DTYPE_F16 && dtype != SBDA_DTYPE_BF16) return SBDA_ERR_DTYPE;
  if (!block_dims_ok(dtype, rows, dim)) return SBDA_ERR_INVALID;
  if (rows == 0) return SBDA_OK;
  if (!x || !weight || !y || !rstd || (residual_add && !x1_out)) return SBDA_ERR_INVALID;
  if (!aligned16(x) || !aligned16(y) || (residual_add && (!aligned16(residual_add) || !aligned16(x1_out))))
    return SBDA_ERR_INVALID;
  BlockNormParams p;
  memset(&p, 0, sizeof(p));
  p.rows = rows;
  p.dim = (int)dim;
  p.eps = eps;
  p.x = x;
  p.add = residual_add;
  p.mask = row_mask;
  p.w = weight;
  p.x1 = x1_out;
  p.y = y;
  p.rstd = rstd;
  return norm_dispatch(dtype, true, p, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int64_t sbda_b200_rms_norm_workspace_floats(int64_t rows, int64_t dim) {
  if (rows < 0 || dim <= 0) return 0;
  return (int64_t)block_ctas(rows) * dim;
}

extern "C" int sbda_b200_rms_norm_backward(int dtype, int64_t rows, int64_t dim, const void* x1,
                                           const float* rstd, const float* weight, const void* grad_y,
                                           const void* grad_x1, const uint8_t* row_mask, void* grad_x,
                                           void* grad_residual, float* grad_weight, float* workspace,
                                           int64_t workspace_floats, void* stream) {
  if (dtype != SBDA_DTYPE_F32 && dtype != SBDA_DTYPE_F16 && dtype != SBDA_DTYPE_BF16) return SBDA_ERR_DTYPE;
  if (!block_dims_ok(dtype, rows, dim)) return SBDA_ERR_INVALID;
  if (!grad_weight) return SBDA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rows == 0) return cudaMemsetAsync(grad_weight, 0, dim * sizeof(float), st) == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
  if (!x1 || !rstd || !weight || !grad_y || !grad_x || !workspace) return SBDA_ERR_INVALID;
  const int ctas = block_ctas(rows);
  if (workspace_floats < (int64_t)ctas * dim) return SBDA_ERR_INVALID;
  if (!aligned16(x1) || !aligned16(grad_y) || !aligned16(grad_x) || (grad_x1 && !aligned16(grad_x1)) ||
      (grad_residual && !aligned16(grad_residual)))
    return SBDA_ERR_INVALID;
  BlockNormParams p;
  memset(&p, 0, sizeof(p));
  p.rows = rows;
  p.dim = (int)dim;
  p.x = x1;
  p.mask = row_mask;
  p.w = weight;
  p.rstd = const_cast<float*>(rstd);
  p.dy = grad_y;
  p.dx1_ext = grad_x1;
  p.dx = grad_x;
  p.dadd = grad_residual;
  p.partial = workspace;
  const int st1 = norm_dispatch(dtype, false, p, st);
  if (st1 != SBDA_OK) return st1;
  sbda_block_weight_reduce_kernel<<<(unsigned)((dim + 127) / 128), 128, 0, st>>>(workspace, ctas, (int)dim,
                                                                                grad_weight);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

namespace {
template <typename TE>
int silu_launch(bool fwd, int64_t n, const void* g, const void* u, const void* dh, void* a, void* b,
                cudaStream_t st) {
  const long long n8 = n / 8;
  const long long want = (n8 + 255) / 256;
  const unsigned grid = (unsigned)(want < 148LL * 16 ? (want > 0 ? want : 1) : 148LL * 16);
  if (fwd)
    sbda_silu_mul_fwd_kernel<TE><<<grid, 256, 0, st>>>(n8, static_cast<const TE*>(g), static_cast<const TE*>(u),
                                                       static_cast<TE*>(a));
  else
    sbda_silu_mul_bwd_kernel<TE><<<grid, 256, 0, st>>>(n8, static_cast<const TE*>(g), static_cast<const TE*>(u),
                                                       static_cast<const TE*>(dh), static_cast<TE*>(a),
                                                       static_cast<TE*>(b));
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

int silu_dispatch(int dtype, bool fwd, int64_t n, const void* g, const void* u, const void* dh, void* a, void* b,
                  cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return silu_launch<float>(fwd, n, g, u, dh, a, b, st);
  if (dtype == SBDA_DTYPE_F16) return silu_launch<__half>(fwd, n, g, u, dh, a, b, st);
  return silu_launch<__nv_bfloat16>(fwd, n, g, u, dh, a, b, st);
}
}  // namespace

extern "C" int sbda_b200_silu_mul_forward(int dtype, int64_t n, const void* gate, const void* up, void* h,
                                          void* stream) {
  if (dtype != SBDA_DTYPE_F32 && dtype != SBDA_DTYPE_F16 && dtype != SBDA_DTYPE_BF16) return SBDA_ERR_DTYPE;
  if (n < 0 || n % 8) return SBDA_ERR_INVALID;
  if (n == 0) return SBDA_OK;
  if (!gate || !up || !h || !aligned16(gate) || !aligned16(up) || !aligned16(h)) return SBDA_ERR_INVALID;
  return silu_dispatch(dtype, true, n, gate, up, nullptr, h, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sbda_b200_silu_mul_backward(int dtype, int64_t n, const void* gate, const void* up,
                                           const void* grad_h, void* grad_gate, void* grad_up, void* stream) {
  if (dtype != SBDA_DTYPE_F32 && dtype != SBDA_DTYPE_F16 && dtype != SBDA_DTYPE_BF16) return SBDA_ERR_DTYPE;
  if (n < 0 || n % 8) return SBDA_ERR_INVALID;
  if (n == 0) return SBDA_OK;
  if (!gate || !up || !grad_h || !grad_gate || !grad_up) return SBDA_ERR_INVALID;
  if (!aligned16(gate) || !aligned16(up) || !aligned16(grad_h) || !aligned16(grad_gate) || !aligned16(grad_up))
    return SBDA_ERR_INVALID;
  return silu_dispatch(dtype, false, n, gate, up, grad_h, grad_gate, grad_up,
                       reinterpret_cast<cudaStream_t>(stream));
}
