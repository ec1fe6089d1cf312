// sbda_v2_normed.cu -- launchers of the windowed kernels with the per-head
// RMSNorm + RoPE of q and k fused into their loads (the NR instances of
// sbda_v2_kernels.cuh), and the fixed-order reduction of their per-CTA
// norm-weight gradients.
//
// Served: head_dim 64, 8 lanes per row (bf16, fp16, fp32), MHA, copy-engine
// layouts, one GPU, and the specialised source sets of the SBDA family:
// {0, 1}, {0, 2}, {0, 1, 2, d} (every walk mode).

#include "sbda_v2_kernels.cuh"

namespace sbda {

template <typename TE, int SHAPE>
int launch_fwd_nr(const FwdMaps& maps, const FwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  auto kern = sbda_fwd_v2_kernel<TE, 8, true, SHAPE, FwdMaps, true>;
  const size_t smem = pl.smem_fwd - (size_t)v2_tile(8) * pl.pitch;  // Q rows stay in registers
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SBDA_ERR_CUDA;
  const long long blocks = (long long)p.B * p.H * pl.g.nT;
  return launch_chained(kern, (unsigned)blocks, smem, st, maps, p) == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE, int SHAPE>
int launch_bwd_nr(const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  auto kern = sbda_bwd_v2_kernel<TE, 8, true, SHAPE, BwdMaps, true>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem_bwd) != cudaSuccess)
    return SBDA_ERR_CUDA;
  return launch_chained(kern, pl.blocks_bwd, pl.smem_bwd, st, maps, p) == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE>
int fwd_nr_shape(const FwdMaps& maps, const FwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  switch (fwd_shape(pl.g, pl.tile)) {
    case 1: return launch_fwd_nr<TE, 1>(maps, p, pl, st);
    case 2: return launch_fwd_nr<TE, 2>(maps, p, pl, st);
    case 3: return launch_fwd_nr<TE, 3>(maps, p, pl, st);
    case 4: return launch_fwd_nr<TE, 4>(maps, p, pl, st);
    default: return SBDA_ERR_UNSUPPORTED;
  }
}

template <typename TE>
int bwd_nr_shape(const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  switch (bwd_shape(pl.g)) {
    case 1: return launch_bwd_nr<TE, 1>(maps, p, pl, st);
    case 2: return launch_bwd_nr<TE, 2>(maps, p, pl, st);
    case 3: return launch_bwd_nr<TE, 3>(maps, p, pl, st);
    case 4: return launch_bwd_nr<TE, 4>(maps, p, pl, st);
    case 5: return launch_bwd_nr<TE, 5>(maps, p, pl, st);
    default: return SBDA_ERR_UNSUPPORTED;
  }
}

bool v2_normed_plan_ok(const V2Plan& pl) {
  return pl.lpr == 8 && fwd_shape(pl.g, pl.tile) != 0 && bwd_shape(pl.g) != 0;
}

int v2_forward_normed(int dtype, const FwdMaps& maps, const FwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  if (!v2_normed_plan_ok(pl)) return SBDA_ERR_UNSUPPORTED;
  if (dtype == SBDA_DTYPE_F32) return fwd_nr_shape<float>(maps, p, pl, st);
  if (dtype == SBDA_DTYPE_F16) return fwd_nr_shape<__half>(maps, p, pl, st);
  return fwd_nr_shape<__nv_bfloat16>(maps, p, pl, st);
}

// Weight-gradient partials: [blocks, 128] (q columns 0..63, k columns 64..127).
// Level 1: CTA k sums rows [256k, 256k + 256) in row order; level 2: one CTA
// sums the level-1 rows in order.  Fixed order, so results are reproducible.
constexpr int kDwRowsPerCta = 256;

__global__ void __launch_bounds__(128) sbda_dw_reduce_rows_kernel(const float* partial, int rows, float* level1) {
  const int t = threadIdx.x;
  const int lo = blockIdx.x * kDwRowsPerCta, hi = min(rows, lo + kDwRowsPerCta);
  float sum = 0.f;
  for (int r = lo; r < hi; ++r) sum += partial[(long long)r * 128 + t];
  level1[blockIdx.x * 128 + t] = sum;
}

__global__ void __launch_bounds__(128) sbda_dw_reduce_final_kernel(const float* level1, int n1, float* grad_q_w,
                                                                    float* grad_k_w) {
  const int t = threadIdx.x;
  float sum = 0.f;
  for (int r = 0; r < n1; ++r) sum += level1[r * 128 + t];
  if (t < 64) grad_q_w[t] = sum;
  else grad_k_w[t - 64] = sum;
}

int64_t v2_normed_workspace_floats(unsigned blocks) {
  const int64_t n1 = ((int64_t)blocks + kDwRowsPerCta - 1) / kDwRowsPerCta;
  return (int64_t)blocks * 128 + n1 * 128;
}

int v2_backward_normed(int dtype, const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl, float* grad_q_w,
                       float* grad_k_w, float* workspace, cudaStream_t st) {
  if (!v2_normed_plan_ok(pl)) return SBDA_ERR_UNSUPPORTED;
  int rc;
  if (dtype == SBDA_DTYPE_F32) rc = bwd_nr_shape<float>(maps, p, pl, st);
  else if (dtype == SBDA_DTYPE_F16) rc = bwd_nr_shape<__half>(maps, p, pl, st);
  else rc = bwd_nr_shape<__nv_bfloat16>(maps, p, pl, st);
  if (rc != SBDA_OK) return rc;
  const int rows = (int)pl.blocks_bwd;
  const int n1 = (rows + kDwRowsPerCta - 1) / kDwRowsPerCta;
  float* level1 = workspace + (int64_t)rows * 128;
  sbda_dw_reduce_rows_kernel<<<n1, 128, 0, st>>>(workspace, rows, level1);
  sbda_dw_reduce_final_kernel<<<1, 128, 0, st>>>(level1, n1, grad_q_w, grad_k_w);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

}  // namespace sbda
