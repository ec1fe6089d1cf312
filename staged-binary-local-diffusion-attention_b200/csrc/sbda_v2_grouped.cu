// sbda_v2_grouped.cu -- grouped-query attention (H query heads sharing Hkv
// kv heads) on the windowed backward.
//
// Each query head h runs the windowed walk of sbda_v2_kernels.cuh with K/V
// staged from kv head h / G and writes its dK / dV contributions as fp32
// partials to a caller workspace [2][B, H, L, D] (the TO = float instances).
// A second kernel sums the G partials of every kv head in head order and
// rounds once to the element type: deterministic, with the accuracy of an
// in-kernel fp32 sum.  The reference's GQA op sums over the group with
// atomics (BiAttn/sbda_triton.py:1363-1434, kernels :803-1065).
//
// Served: 8 lanes per row (head_dim <= 64, a multiple of 8), the SBDA
// family's specialised source sets, copy-engine layouts, one GPU.  Other
// calls return SBDA_ERR_UNSUPPORTED before launching anything, and the caller
// runs the general kernels.

#include "sbda_v2_kernels.cuh"

namespace sbda {

template <typename TE, int SHAPE>
int launch_bwd_grouped(const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  auto kern = sbda_bwd_v2_kernel<TE, 8, true, SHAPE, BwdMaps, false, float>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem_bwd) != cudaSuccess)
    return SBDA_ERR_CUDA;
  return launch_chained(kern, pl.blocks_bwd, pl.smem_bwd, st, maps, p) == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE>
int bwd_grouped_shape(const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  switch (bwd_shape(pl.g)) {
    case 1: return launch_bwd_grouped<TE, 1>(maps, p, pl, st);
    case 2: return launch_bwd_grouped<TE, 2>(maps, p, pl, st);
    case 3: return launch_bwd_grouped<TE, 3>(maps, p, pl, st);
    case 4: return launch_bwd_grouped<TE, 4>(maps, p, pl, st);
    case 5: return launch_bwd_grouped<TE, 5>(maps, p, pl, st);
    default: return SBDA_ERR_UNSUPPORTED;
  }
}

bool v2_grouped_plan_ok(const V2Plan& pl) { return pl.lpr == 8 && bwd_shape(pl.g) != 0; }

// out[b, hk, l, :] = sum over g < G (in order) of part[b, hk * G + g, l, :];
// part is a contiguous fp32 [B, H, L, D] array, out a [B, Hkv, L, D] view.
// One thread per 8 channels of a row; blockIdx.y picks dK (0) or dV (1).
template <typename TE>
__global__ void __launch_bounds__(256) sbda_kv_group_sum_kernel(const float* __restrict__ partial, long long part_stride,
                                                                int Hkv, int G, int L, int D, TensorArg dk, TensorArg dv) {
  const int chunks = D / 8;
  const long long item = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.z;
  if (item >= (long long)Hkv * L * chunks) return;
  const int chunk = (int)(item % chunks);
  const long long row = item / chunks;  // (hk, l) within batch entry b
  const int l = (int)(row % L);
  const int hk = (int)(row / L);
  const float* src = partial + blockIdx.y * part_stride;
  const int H = Hkv * G;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int g = 0; g < G; ++g) {
    const float* r = src + (((long long)b * H + (long long)hk * G + g) * L + l) * D + chunk * 8;
    const float4 x = *reinterpret_cast<const float4*>(r);
    const float4 y = *reinterpret_cast<const float4*>(r + 4);
    acc[0] += x.x;
    acc[1] += x.y;
    acc[2] += x.z;
    acc[3] += x.w;
    acc[4] += y.x;
    acc[5] += y.y;
    acc[6] += y.z;
    acc[7] += y.w;
  }
  const TensorArg& t = blockIdx.y == 0 ? dk : dv;
  TE* dst = reinterpret_cast<TE*>(const_cast<void*>(t.ptr)) + (long long)b * t.sb + (long long)hk * t.sh +
            (long long)l * t.sl + (long long)chunk * 8 * t.sd;
#pragma unroll
  for (int e = 0; e < 8; ++e) dst[(long long)e * t.sd] = Elem<TE>::from_float(acc[e]);
}

template <typename TE>
int group_sum(const float* workspace, const BwdV2Params& p, int Hkv, const TensorArg& dk, const TensorArg& dv,
              cudaStream_t st) {
  const long long items = (long long)Hkv * p.L * (p.D / 8);
  const dim3 grid((unsigned)((items + 255) / 256), 2, (unsigned)p.B);
  const long long part_stride = (long long)p.B * p.H * p.L * p.D;
  sbda_kv_group_sum_kernel<TE><<<grid, 256, 0, st>>>(workspace, part_stride, Hkv, p.G, p.L, p.D, dk, dv);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

int v2_backward_grouped(int dtype, const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl, const float* workspace,
                        int Hkv, const TensorArg& dk, const TensorArg& dv, cudaStream_t st) {
  if (!v2_grouped_plan_ok(pl) || p.D % 8) return SBDA_ERR_UNSUPPORTED;
  int rc;
  if (dtype == SBDA_DTYPE_F32) rc = bwd_grouped_shape<float>(maps, p, pl, st);
  else if (dtype == SBDA_DTYPE_F16) rc = bwd_grouped_shape<__half>(maps, p, pl, st);
  else rc = bwd_grouped_shape<__nv_bfloat16>(maps, p, pl, st);
  if (rc != SBDA_OK) return rc;
  if (dtype == SBDA_DTYPE_F32) return group_sum<float>(workspace, p, Hkv, dk, dv, st);
  if (dtype == SBDA_DTYPE_F16) return group_sum<__half>(workspace, p, Hkv, dk, dv, st);
  return group_sum<__nv_bfloat16>(workspace, p, Hkv, dk, dv, st);
}

}  // namespace sbda
