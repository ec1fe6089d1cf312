// sbda_v2.cu -- launchers of the windowed SBDA kernels (sbda_v2_kernels.cuh)
// on plain q/k/v: source-set shape dispatch per dtype and lanes per row.

#include "sbda_v2_kernels.cuh"

namespace sbda {

// --------------------------------------------------------------------------
// Launchers
// --------------------------------------------------------------------------

template <typename TE, int LPR, bool TMA, int SHAPE, typename Maps>
int launch_fwd_v2(const Maps& maps, const FwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  auto kern = sbda_fwd_v2_kernel<TE, LPR, TMA, SHAPE, Maps>;
  // The copy-engine path keeps Q out of shared memory.
  const size_t smem = pl.smem_fwd - (TMA ? (size_t)v2_tile(LPR) * pl.pitch : 0);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SBDA_ERR_CUDA;
  const long long blocks = (long long)p.B * p.H * pl.g.nT;
  return launch_chained(kern, (unsigned)blocks, smem, st, maps, p) == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE, int LPR, bool TMA, int SHAPE, typename Maps>
int launch_bwd_v2(const Maps& maps, const BwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  auto kern = sbda_bwd_v2_kernel<TE, LPR, TMA, SHAPE, Maps>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem_bwd) != cudaSuccess)
    return SBDA_ERR_CUDA;
  return launch_chained(kern, pl.blocks_bwd, pl.smem_bwd, st, maps, p) == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE, bool TMA, typename Maps>
int fwd_v2_lpr(const Maps& maps, const FwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  if constexpr (TMA) {
    if (pl.lpr == 8) {
      const V2Geometry& g = pl.g;
      if (g.has0 && g.has1 && !g.has2 && !g.has_far) return launch_fwd_v2<TE, 8, TMA, 1>(maps, p, pl, st);
      if (g.has0 && !g.has1 && g.has2 && !g.has_far) return launch_fwd_v2<TE, 8, TMA, 2>(maps, p, pl, st);
      if (g.has0 && g.has1 && g.has2 && g.has_far)
        return g.d < pl.tile ? launch_fwd_v2<TE, 8, TMA, 4>(maps, p, pl, st) : launch_fwd_v2<TE, 8, TMA, 3>(maps, p, pl, st);
    }
  }
  if constexpr (sizeof(TE) == 4) {
    if (pl.lpr == 4) return launch_fwd_v2<TE, 4, TMA, 0>(maps, p, pl, st);
  }
  if (pl.lpr == 8) return launch_fwd_v2<TE, 8, TMA, 0>(maps, p, pl, st);
  if (pl.lpr == 16) return launch_fwd_v2<TE, 16, TMA, 0>(maps, p, pl, st);
  return SBDA_ERR_UNSUPPORTED;
}

template <typename TE, bool TMA, typename Maps>
int bwd_v2_lpr(const Maps& maps, const BwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  // Specialised shapes are compiled for the copy-engine path at 8 lanes per row.
  if constexpr (TMA) {
    if (pl.lpr == 8) {
      switch (bwd_shape(pl.g)) {
        case 1: return launch_bwd_v2<TE, 8, TMA, 1>(maps, p, pl, st);
        case 2: return launch_bwd_v2<TE, 8, TMA, 2>(maps, p, pl, st);
        case 3: return launch_bwd_v2<TE, 8, TMA, 3>(maps, p, pl, st);
        case 4: return launch_bwd_v2<TE, 8, TMA, 4>(maps, p, pl, st);
        case 5: return launch_bwd_v2<TE, 8, TMA, 5>(maps, p, pl, st);
        default: break;
      }
    }
  }
  if constexpr (sizeof(TE) == 4) {
    if (pl.lpr == 4) return launch_bwd_v2<TE, 4, TMA, 0>(maps, p, pl, st);
  }
  if (pl.lpr == 8) return launch_bwd_v2<TE, 8, TMA, 0>(maps, p, pl, st);
  if (pl.lpr == 16) return launch_bwd_v2<TE, 16, TMA, 0>(maps, p, pl, st);
  return SBDA_ERR_UNSUPPORTED;
}

template <bool TMA, typename Maps>
int fwd_v2_dtype(int dtype, const Maps& maps, const FwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return fwd_v2_lpr<float, TMA>(maps, p, pl, st);
  if (dtype == SBDA_DTYPE_F16) return fwd_v2_lpr<__half, TMA>(maps, p, pl, st);
  return fwd_v2_lpr<__nv_bfloat16, TMA>(maps, p, pl, st);
}

template <bool TMA, typename Maps>
int bwd_v2_dtype(int dtype, const Maps& maps, const BwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return bwd_v2_lpr<float, TMA>(maps, p, pl, st);
  if (dtype == SBDA_DTYPE_F16) return bwd_v2_lpr<__half, TMA>(maps, p, pl, st);
  return bwd_v2_lpr<__nv_bfloat16, TMA>(maps, p, pl, st);
}

int v2_forward(int dtype, bool tma, const FwdMaps& maps, const FwdV2Params& p, const V2Plan& pl, cudaStream_t st) {
  return tma ? fwd_v2_dtype<true>(dtype, maps, p, pl, st) : fwd_v2_dtype<false>(dtype, maps, p, pl, st);
}

int v2_backward(int dtype, bool tma, const BwdMaps& maps, const BwdV2Params& p, const V2Plan& pl,
                cudaStream_t st) {
  return tma ? bwd_v2_dtype<true>(dtype, maps, p, pl, st) : bwd_v2_dtype<false>(dtype, maps, p, pl, st);
}

// Sequence shards: one tensor map per rank, copy-engine layouts only.
int v2_forward_sharded(int dtype, const ShardFwdMaps& maps, const FwdV2Params& p, const V2Plan& pl,
                       cudaStream_t st) {
  return fwd_v2_dtype<true>(dtype, maps, p, pl, st);
}

int v2_backward_sharded(int dtype, const ShardBwdMaps& maps, const BwdV2Params& p, const V2Plan& pl,
                        cudaStream_t st) {
  return bwd_v2_dtype<true>(dtype, maps, p, pl, st);
}

}  // namespace sbda
