// sbda_v3.cu -- uniform SBDA kernels: any 1..4 distinct offsets, any number
// of them far apart, native GQA, any head size <= 128.
//
// Same function as the reference's fused ops (BiAttn/sbda_triton.py:1290-1360
// forward O and softmax statistics, gather backward; 1363-1434 GQA) and their
// eager oracle (BiAttn/left_v2.py:335-405).  The reference accepts any two or
// four offsets; the windowed (sbda_v2.cu) and general (sbda_v1.cu) kernels
// stage one near window plus at most one far tile, so schedules with several
// far offsets (butterfly, radix4, mesh at large strides, ...) land here.
//
//  * Every source is its own shifted tile: for the tile of positions
//    [i0, i0 + T), source s reads K/V rows [i0 - o_s, i0 - o_s + T), staged
//    by TMA (zero fill before 0 and past L).  Row r of every staged tile
//    belongs to row r of the tile, so a row group only reads its own rows.
//  * Backward, key-centric and atomic-free: the CTA of key tile j (one kv
//    head, looping over its query heads) visits, for each source s, the
//    consumer tile [j0 + o_s, j0 + o_s + T) with all of that tile's sources,
//    recomputes the consumer softmax from the saved LSE, and adds source s's
//    terms to the keys of tile j (same local row).  The visit with the
//    smallest offset also writes the consumers' dQ, so every query row is
//    written once; rows below the smallest offset have no source and get
//    dQ = 0.
//  Each consumer softmax is formed once per source (S times), the price of
//  serving arbitrary offset sets without cross-tile records.
//  * An optional per-row source mask (uint8 [B, L], bit s allows source s of
//    that row) restricts the sources further: padding holes and segment
//    resets, as the reference's eager path builds them (left_v2.py:349-373).

#include "sbda_common.cuh"

namespace sbda {

template <typename TE, int LPR, bool TMA>
__global__ void __launch_bounds__(kThreads) sbda_fwd_v3_kernel(const __grid_constant__ FwdMaps maps,
                                                               const V3Params p) {
  constexpr int T = v2_tile(LPR);
  constexpr int P = LPR * FragIO<TE>::kLaneBytes;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int grp = tid / LPR, l = tid % LPR;
  int bid = blockIdx.x;
  const int h = bid % p.H;
  bid /= p.H;
  const int t = bid % p.nT;
  const int b = bid / p.nT;
  const int hk = h / p.G;
  const int i0 = t * T;
  const int S = p.S;

  uint8_t* Qs = smem;
  uint8_t* Ks = Qs + T * P;      // S tiles; source s at Ks + s * T * P
  uint8_t* Vs = Ks + S * T * P;
  uint64_t* bar = reinterpret_cast<uint64_t*>(Vs + S * T * P);

  if constexpr (TMA) {
    if (tid == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
      mbar_arrive_expect_tx(bar, (uint32_t)((1 + 2 * S) * T * P));
      tma_rows(Qs, &maps.qT, bar, p.slots_q, i0, h, b);
      for (int s = 0; s < S; ++s) {
        tma_rows(Ks + s * T * P, &maps.kT, bar, p.slots_k, i0 - p.off[s], hk, b);
        tma_rows(Vs + s * T * P, &maps.vT, bar, p.slots_v, i0 - p.off[s], hk, b);
      }
    }
    const bool ok = mbar_wait_bounded(bar, 0);
    if (__syncthreads_or(!ok)) {
      fault_and_drain(p.status, bar, 0);
      return;
    }
  } else {
    constexpr int PE = P / sizeof(TE);
    generic_rows<TE>(Qs, p.q, b, h, i0, T, p.L, p.D, PE);
    for (int s = 0; s < S; ++s) {
      generic_rows<TE>(Ks + s * T * P, p.k, b, hk, i0 - p.off[s], T, p.L, p.D, PE);
      generic_rows<TE>(Vs + s * T * P, p.v, b, hk, i0 - p.off[s], T, p.L, p.D, PE);
    }
    __syncthreads();
  }

  const float c1 = p.scale * kLog2e;
  TE* out = reinterpret_cast<TE*>(const_cast<void*>(p.out.ptr)) + (long long)b * p.out.sb +
            (long long)h * p.out.sh;
  float* lse = p.lse + ((long long)b * p.H + h) * p.L;
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    const int r = grp * 4 + i, pos = i0 + r;
    const Frag q = FragIO<TE>::load(Qs + r * P, l);
    const unsigned allow = p.mask ? (pos < p.L ? p.mask[(long long)b * p.L + pos] : 0u) : 0xFu;
    float sc[4];
    float m = -INFINITY;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      sc[s] = -INFINITY;
      if (s < S) {
        const float a = lane_group_sum<LPR>(frag_dot(q, FragIO<TE>::load(Ks + (s * T + r) * P, l)));
        if (pos - p.off[s] >= 0 && ((allow >> s) & 1u)) sc[s] = a * c1;  // log2 units
      }
      m = fmaxf(m, sc[s]);
    }
    const bool any = m != -INFINITY;
    float e[4], sum = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      e[s] = sc[s] != -INFINITY ? fast_exp2(sc[s] - m) : 0.f;
      sum += e[s];
    }
    const float inv = any ? __frcp_rn(sum) : 0.f;
    Frag o = frag_zero();
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (s < S) frag_axpy(o, e[s] * inv, FragIO<TE>::load(Vs + (s * T + r) * P, l));
    if (pos < p.L) {
      store_frag<TE, TMA>(out + (long long)pos * p.out.sl, p.out.sd, p.D, l, o);
      if (l == 0) lse[pos] = any ? (m + __log2f(sum)) * kLn2 : -INFINITY;
    }
  }
}

template <typename TE, int LPR, bool TMA>
__global__ void __launch_bounds__(kThreads, 2) sbda_bwd_v3_kernel(const __grid_constant__ BwdMaps maps,
                                                                  const V3Params p) {
  constexpr int T = v2_tile(LPR);
  constexpr int P = LPR * FragIO<TE>::kLaneBytes;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int grp = tid / LPR, l = tid % LPR;
  int bid = blockIdx.x;
  const int hk = bid % p.Hkv;
  bid /= p.Hkv;
  const int t = bid % p.nT;
  const int b = bid / p.nT;
  const int j0 = t * T;
  const int S = p.S;
  const int a = grp * 4;

  uint8_t* Qc = smem;            // consumer tile: Q rows
  uint8_t* Dc = Qc + T * P;      // consumer tile: dO rows
  uint8_t* Ks = Dc + T * P;      // the consumer tile's S source tiles
  uint8_t* Vs = Ks + S * T * P;
  uint64_t* bar = reinterpret_cast<uint64_t*>(Vs + S * T * P);
  if constexpr (TMA) {
    if (tid == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
    }
    __syncthreads();
  }

  const float scale = p.scale;
  const float c1 = scale * kLog2e;
  Frag dk_acc[4], dv_acc[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) dk_acc[i] = dv_acc[i] = frag_zero();

  uint32_t phase = 0;
#pragma unroll 1
  for (int gi = 0; gi < p.G; ++gi) {
    const int h = hk * p.G + gi;
    const float* lse = p.lse + ((long long)b * p.H + h) * p.L;
    TE* dq = reinterpret_cast<TE*>(const_cast<void*>(p.dq.ptr)) + (long long)b * p.dq.sb + (long long)h * p.dq.sh;
#pragma unroll 1
    for (int s = 0; s < S; ++s) {
      const int c0 = j0 + p.off[s];  // consumer tile of source s
      if (c0 >= p.L) continue;       // uniform across the CTA
      __syncthreads();               // the previous visit's readers are done
      if constexpr (TMA) {
        if (tid == 0) {
          mbar_arrive_expect_tx(bar, (uint32_t)((2 + 2 * S) * T * P));
          tma_rows(Qc, &maps.qT, bar, p.slots_q, c0, h, b);
          tma_rows(Dc, &maps.dT, bar, p.slots_d, c0, h, b);
          for (int u = 0; u < S; ++u) {
            tma_rows(Ks + u * T * P, &maps.kT, bar, p.slots_k, c0 - p.off[u], hk, b);
            tma_rows(Vs + u * T * P, &maps.vT, bar, p.slots_v, c0 - p.off[u], hk, b);
          }
        }
        const bool ok = mbar_wait_bounded(bar, phase & 1);
        if (__syncthreads_or(!ok)) {
          fault_and_drain(p.status, bar, phase & 1);
          return;
        }
        ++phase;
      } else {
        constexpr int PE = P / sizeof(TE);
        generic_rows<TE>(Qc, p.q, b, h, c0, T, p.L, p.D, PE);
        generic_rows<TE>(Dc, p.dout, b, h, c0, T, p.L, p.D, PE);
        for (int u = 0; u < S; ++u) {
          generic_rows<TE>(Ks + u * T * P, p.k, b, hk, c0 - p.off[u], T, p.L, p.D, PE);
          generic_rows<TE>(Vs + u * T * P, p.v, b, hk, c0 - p.off[u], T, p.L, p.D, PE);
        }
        __syncthreads();
      }
#pragma unroll 1
      for (int i = 0; i < 4; ++i) {
        const int r = a + i, cpos = c0 + r;
        const bool inr = cpos < p.L;
        const float lq = inr ? lse[cpos] * kLog2e : 0.f;
        const unsigned allow = p.mask ? (inr ? p.mask[(long long)b * p.L + cpos] : 0u) : 0xFu;
        const Frag qf = FragIO<TE>::load(Qc + r * P, l);
        const Frag df = FragIO<TE>::load(Dc + r * P, l);
        float pr[4], bv[4];
        float delta = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          pr[u] = bv[u] = 0.f;
          if (u < S) {
            const float av = lane_group_sum<LPR>(frag_dot(qf, FragIO<TE>::load(Ks + (u * T + r) * P, l)));
            bv[u] = lane_group_sum<LPR>(frag_dot(df, FragIO<TE>::load(Vs + (u * T + r) * P, l)));
            if (inr && cpos - p.off[u] >= 0 && ((allow >> u) & 1u)) pr[u] = fast_exp2(fmaf(av, c1, -lq));
            delta = fmaf(pr[u], bv[u], delta);
          }
        }
        float ds[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) ds[u] = pr[u] * (bv[u] - delta) * scale;
        // Source s of consumer row r is key row r of tile j.
        float dss = ds[0], prs = pr[0];
#pragma unroll
        for (int u = 1; u < 4; ++u)
          if (u == s) dss = ds[u], prs = pr[u];
        frag_axpy(dk_acc[i], dss, qf);
        frag_axpy(dv_acc[i], prs, df);
        if (s == p.s_q && inr) {
          Frag gq = frag_zero();
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (u < S) frag_axpy(gq, ds[u], FragIO<TE>::load(Ks + (u * T + r) * P, l));
          store_frag<TE, TMA>(dq + (long long)cpos * p.dq.sl, p.dq.sd, p.D, l, gq);
        }
      }
    }
    // Query rows below the smallest offset have no source: dQ = 0.
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      const int pos = j0 + a + i;
      if (pos < p.o_min && pos < p.L)
        store_frag<TE, TMA>(dq + (long long)pos * p.dq.sl, p.dq.sd, p.D, l, frag_zero());
    }
  }

  TE* dk = reinterpret_cast<TE*>(const_cast<void*>(p.dk.ptr)) + (long long)b * p.dk.sb + (long long)hk * p.dk.sh;
  TE* dv = reinterpret_cast<TE*>(const_cast<void*>(p.dv.ptr)) + (long long)b * p.dv.sb + (long long)hk * p.dv.sh;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = j0 + a + i;
    if (j < p.L) {
      store_frag<TE, TMA>(dk + (long long)j * p.dk.sl, p.dk.sd, p.D, l, dk_acc[i]);
      store_frag<TE, TMA>(dv + (long long)j * p.dv.sl, p.dv.sd, p.D, l, dv_acc[i]);
    }
  }
}

// --------------------------------------------------------------------------
// Launchers
// --------------------------------------------------------------------------

template <typename TE, int LPR, bool TMA>
int launch_fwd_v3(const FwdMaps& maps, const V3Params& p, const V3Plan& pl, cudaStream_t st) {
  auto kern = sbda_fwd_v3_kernel<TE, LPR, TMA>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem_fwd) != cudaSuccess)
    return SBDA_ERR_CUDA;
  const long long blocks = (long long)p.B * p.H * p.nT;
  kern<<<(unsigned)blocks, kThreads, pl.smem_fwd, st>>>(maps, p);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE, int LPR, bool TMA>
int launch_bwd_v3(const BwdMaps& maps, const V3Params& p, const V3Plan& pl, cudaStream_t st) {
  auto kern = sbda_bwd_v3_kernel<TE, LPR, TMA>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem_bwd) != cudaSuccess)
    return SBDA_ERR_CUDA;
  const long long blocks = (long long)p.B * p.Hkv * p.nT;
  kern<<<(unsigned)blocks, kThreads, pl.smem_bwd, st>>>(maps, p);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE, bool TMA>
int v3_dispatch(bool fwd, const void* maps, const V3Params& p, const V3Plan& pl, cudaStream_t st) {
  if constexpr (sizeof(TE) == 4) {
    if (pl.lpr == 4)
      return fwd ? launch_fwd_v3<TE, 4, TMA>(*static_cast<const FwdMaps*>(maps), p, pl, st)
                 : launch_bwd_v3<TE, 4, TMA>(*static_cast<const BwdMaps*>(maps), p, pl, st);
  }
  if (pl.lpr == 8)
    return fwd ? launch_fwd_v3<TE, 8, TMA>(*static_cast<const FwdMaps*>(maps), p, pl, st)
               : launch_bwd_v3<TE, 8, TMA>(*static_cast<const BwdMaps*>(maps), p, pl, st);
  if (pl.lpr == 16)
    return fwd ? launch_fwd_v3<TE, 16, TMA>(*static_cast<const FwdMaps*>(maps), p, pl, st)
               : launch_bwd_v3<TE, 16, TMA>(*static_cast<const BwdMaps*>(maps), p, pl, st);
  return SBDA_ERR_UNSUPPORTED;
}

template <bool TMA>
int v3_dtype(int dtype, bool fwd, const void* maps, const V3Params& p, const V3Plan& pl, cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return v3_dispatch<float, TMA>(fwd, maps, p, pl, st);
  if (dtype == SBDA_DTYPE_F16) return v3_dispatch<__half, TMA>(fwd, maps, p, pl, st);
  return v3_dispatch<__nv_bfloat16, TMA>(fwd, maps, p, pl, st);
}

int v3_forward(int dtype, bool tma, const FwdMaps& maps, const V3Params& p, const V3Plan& pl, cudaStream_t st) {
  return tma ? v3_dtype<true>(dtype, true, &maps, p, pl, st) : v3_dtype<false>(dtype, true, &maps, p, pl, st);
}

int v3_backward(int dtype, bool tma, const BwdMaps& maps, const V3Params& p, const V3Plan& pl, cudaStream_t st) {
  return tma ? v3_dtype<true>(dtype, false, &maps, p, pl, st) : v3_dtype<false>(dtype, false, &maps, p, pl, st);
}

}  // namespace sbda
