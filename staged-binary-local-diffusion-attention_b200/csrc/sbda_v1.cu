// sbda_v1.cu -- general SBDA kernels: any 1..4 offsets with at most one beyond
// the tile (near window + one far tile), native GQA, any head size <= 128.
//
// Forward and gather-form backward of the exact-source attention of the
// reference (BiAttn/sbda_triton.py:134-201 block forward, :440-503 weights,
// :506-587 dQ, :590-671 key-centric dK/dV; eager form BiAttn/left_v2.py:335-405).
//
//  * One CTA owns a tile of TILE consecutive positions of one (batch, head).
//    Rows are staged in shared memory by TMA (cp.async.bulk.tensor, no
//    multicast) from 4-D tensor maps over the caller's strided [B,H,L,D]
//    view; rows before position 0 or past L are zero-filled by the copy
//    engine and scores are masked explicitly (i - o >= 0).
//  * Offsets split into a near window (o <= TILE, a left halo of Hn rows)
//    and at most one far offset f with its own tile; when f is a multiple of
//    TILE, tiles launch in chain order t, t+f/TILE, ... so the far tile is the
//    L2-resident tile of the previous CTA.
//  * The backward is gather form and atomic-free: the CTA of key tile
//    [j0, j0+TILE) recomputes the softmax of every consumer of its keys
//    ([j0, j0+TILE+Hn) and [j0+f, j0+f+TILE)) and writes dQ / dK / dV once.
//    Native GQA: the CTA owns a kv head and loops over its query heads.
// The windowed kernels of sbda_v2.cu replace these for the MHA schedules
// they serve; these remain the general path.

#include "sbda_common.cuh"

namespace sbda {

// --------------------------------------------------------------------------
// Forward
// --------------------------------------------------------------------------

template <typename TE, int NV, int TILE, bool TMA, typename Maps = FwdMaps>
__global__ void __launch_bounds__(kThreads) sbda_fwd_kernel(const __grid_constant__ Maps maps,
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
  const int i0 = t * TILE;          // local tile start
  const int i0g = p.sh.pos0 + i0;   // its global position
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
      int c;
      tma_rows(Qs, &maps.qT, bar, p.slots_q, i0, h, b);
      if (Hn > 0) {
        tma_rows(Kn, pick_map(maps.kH, p.sh, i0g - Hn, c), bar, p.slots_k, c, hk, b);
        tma_rows(Vn, pick_map(maps.vH, p.sh, i0g - Hn, c), bar, p.slots_v, c, hk, b);
      }
      tma_rows(Kn + Hn * P, pick_map(maps.kT, p.sh, i0g, c), bar, p.slots_k, c, hk, b);
      tma_rows(Vn + Hn * P, pick_map(maps.vT, p.sh, i0g, c), bar, p.slots_v, c, hk, b);
      if (g.has_far) {
        tma_rows(Kf, pick_map(maps.kT, p.sh, i0g - g.f, c), bar, p.slots_k, c, hk, b);
        tma_rows(Vf, pick_map(maps.vT, p.sh, i0g - g.f, c), bar, p.slots_v, c, hk, b);
      }
    }
    const bool ok = mbar_wait_bounded(bar, 0);
    if (__syncthreads_or(!ok)) {
      fault_and_drain(p.status, bar, 0);
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
    const int i = i0g + r;  // global position (masks); stores use the local row i0 + r
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
    const int il = i0 + r;
    if (il < p.L) {
      TE* orow = out + (long long)b * p.out.sb + (long long)h * p.out.sh + (long long)il * p.out.sl;
      store_row<TE, NV, TMA>(orow, p.out.sd, p.D, l8, of);
      if (l8 == 0) lse[il] = sum > 0.f ? mx + __logf(sum) : -INFINITY;
    }
  }
}

// --------------------------------------------------------------------------
// Backward (gather form)
// --------------------------------------------------------------------------

template <typename TE, int NV, int TILE, bool TMA, typename Maps = BwdMaps>
__global__ void __launch_bounds__(kThreads) sbda_bwd_kernel(const __grid_constant__ Maps maps,
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
  const int j0 = t * TILE;          // local tile start
  const int j0g = p.sh.pos0 + j0;   // its global position
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
        int c;
        tma_rows(QN, pick_map(maps.qT, p.sh, j0g, c), bar, p.slots_q, c, h, b);
        tma_rows(DN, pick_map(maps.dT, p.sh, j0g, c), bar, p.slots_d, c, h, b);
        if (Hn > 0) {
          tma_rows(QN + TILE * P, pick_map(maps.qH, p.sh, j0g + TILE, c), bar, p.slots_q, c, h, b);
          tma_rows(DN + TILE * P, pick_map(maps.dH, p.sh, j0g + TILE, c), bar, p.slots_d, c, h, b);
        }
        if (far) {
          tma_rows(QF, pick_map(maps.qT, p.sh, j0g + f, c), bar, p.slots_q, c, h, b);
          tma_rows(DF, pick_map(maps.dT, p.sh, j0g + f, c), bar, p.slots_d, c, h, b);
        }
        if (gi == 0) {
          tma_rows(KN + Hn * P, pick_map(maps.kT, p.sh, j0g, c), bar, p.slots_k, c, hk, b);
          tma_rows(VN + Hn * P, pick_map(maps.vT, p.sh, j0g, c), bar, p.slots_v, c, hk, b);
          if (Hn > 0) {
            tma_rows(KN, pick_map(maps.kH, p.sh, j0g - Hn, c), bar, p.slots_k, c, hk, b);
            tma_rows(VN, pick_map(maps.vH, p.sh, j0g - Hn, c), bar, p.slots_v, c, hk, b);
            tma_rows(KN + (Hn + TILE) * P, pick_map(maps.kH, p.sh, j0g + TILE, c), bar, p.slots_k, c, hk, b);
            tma_rows(VN + (Hn + TILE) * P, pick_map(maps.vH, p.sh, j0g + TILE, c), bar, p.slots_v, c, hk, b);
          }
          if (far) {
            tma_rows(KFL, pick_map(maps.kT, p.sh, j0g - f, c), bar, p.slots_k, c, hk, b);
            tma_rows(VFL, pick_map(maps.vT, p.sh, j0g - f, c), bar, p.slots_v, c, hk, b);
            tma_rows(KFR + Hn * P, pick_map(maps.kT, p.sh, j0g + f, c), bar, p.slots_k, c, hk, b);
            tma_rows(VFR + Hn * P, pick_map(maps.vT, p.sh, j0g + f, c), bar, p.slots_v, c, hk, b);
            if (Hn > 0) {
              tma_rows(KFL + TILE * P, pick_map(maps.kH, p.sh, j0g - f + TILE, c), bar, p.slots_k, c, hk, b);
              tma_rows(VFL + TILE * P, pick_map(maps.vH, p.sh, j0g - f + TILE, c), bar, p.slots_v, c, hk, b);
              tma_rows(KFR, pick_map(maps.kH, p.sh, j0g + f - Hn, c), bar, p.slots_k, c, hk, b);
              tma_rows(VFR, pick_map(maps.vH, p.sh, j0g + f - Hn, c), bar, p.slots_v, c, hk, b);
            }
          }
        }
      }
      const bool ok = mbar_wait_bounded(bar, gi & 1);
      if (__syncthreads_or(!ok)) {
        fault_and_drain(p.status, bar, gi & 1);
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
    const long long bh = (long long)b * p.H + h;
#pragma unroll 1
    for (int base = 0; base < NC; base += kGroups) {
      const bool act = base + grp < NC;
      const int c = act ? base + grp : NC - 1;
      const bool nearc = c < TILE + Hn;
      const int cf = c - (TILE + Hn);
      const int q = nearc ? j0g + c : j0g + f + cf;  // global consumer position
      const bool inr = q < p.sh.total_len;
      const float lq = inr ? lse_at(p.sh, bh, q) : 0.f;
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
        TE* dst = dq_base + (long long)b * p.dq.sb + (long long)h * p.dq.sh + (long long)(j0 + c) * p.dq.sl;
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

template <typename TE, int NV, int TILE, bool TMA, typename Maps = FwdMaps>
int launch_fwd(const Maps& maps, const FwdParams& p, const Plan& pl, cudaStream_t stream) {
  auto kern = sbda_fwd_kernel<TE, NV, TILE, TMA, Maps>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem_fwd) != cudaSuccess)
    return SBDA_ERR_CUDA;
  const long long blocks = (long long)p.B * p.H * pl.g.nT;
  kern<<<(unsigned)blocks, kThreads, pl.smem_fwd, stream>>>(maps, p);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE, int NV, int TILE, bool TMA, typename Maps = BwdMaps>
int launch_bwd(const Maps& maps, const BwdParams& p, const Plan& pl, cudaStream_t stream) {
  auto kern = sbda_bwd_kernel<TE, NV, TILE, TMA, Maps>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem_bwd) != cudaSuccess)
    return SBDA_ERR_CUDA;
  const long long blocks = (long long)p.B * p.Hkv * pl.g.nT;
  kern<<<(unsigned)blocks, kThreads, pl.smem_bwd, stream>>>(maps, p);
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

// Instantiated (pitch, tile) pairs: 128 B -> 64; 256 B -> 64, 32; 512 B -> 32, 16.
#define SBDA_FOR_TILES(LAUNCH, TE, TMA, MAPS, ...)                                        \
  do {                                                                                   \
    if (pl.nv == 1 && pl.tile == 64) return LAUNCH<TE, 1, 64, TMA, MAPS>(__VA_ARGS__);   \
    if (pl.nv == 2 && pl.tile == 64) return LAUNCH<TE, 2, 64, TMA, MAPS>(__VA_ARGS__);   \
    if (pl.nv == 2 && pl.tile == 32) return LAUNCH<TE, 2, 32, TMA, MAPS>(__VA_ARGS__);   \
    if (pl.nv == 4 && pl.tile == 32) return LAUNCH<TE, 4, 32, TMA, MAPS>(__VA_ARGS__);   \
    if (pl.nv == 4 && pl.tile == 16) return LAUNCH<TE, 4, 16, TMA, MAPS>(__VA_ARGS__);   \
    return SBDA_ERR_UNSUPPORTED;                                                         \
  } while (0)

template <typename TE, bool TMA, typename Maps>
int fwd_tiles(const Maps& maps, const FwdParams& p, const Plan& pl, cudaStream_t st) {
  SBDA_FOR_TILES(launch_fwd, TE, TMA, Maps, maps, p, pl, st);
}
template <typename TE, bool TMA, typename Maps>
int bwd_tiles(const Maps& maps, const BwdParams& p, const Plan& pl, cudaStream_t st) {
  SBDA_FOR_TILES(launch_bwd, TE, TMA, Maps, maps, p, pl, st);
}

template <bool TMA, typename Maps>
int fwd_dtype_v1(int dtype, const Maps& maps, const FwdParams& p, const Plan& pl, cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return fwd_tiles<float, TMA, Maps>(maps, p, pl, st);
  if (dtype == SBDA_DTYPE_F16) return fwd_tiles<__half, TMA, Maps>(maps, p, pl, st);
  return fwd_tiles<__nv_bfloat16, TMA, Maps>(maps, p, pl, st);
}
template <bool TMA, typename Maps>
int bwd_dtype_v1(int dtype, const Maps& maps, const BwdParams& p, const Plan& pl, cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return bwd_tiles<float, TMA, Maps>(maps, p, pl, st);
  if (dtype == SBDA_DTYPE_F16) return bwd_tiles<__half, TMA, Maps>(maps, p, pl, st);
  return bwd_tiles<__nv_bfloat16, TMA, Maps>(maps, p, pl, st);
}

int v1_forward(int dtype, bool tma, const FwdMaps& maps, const FwdParams& p, const Plan& pl, cudaStream_t st) {
  return tma ? fwd_dtype_v1<true, FwdMaps>(dtype, maps, p, pl, st)
             : fwd_dtype_v1<false, FwdMaps>(dtype, maps, p, pl, st);
}

int v1_backward(int dtype, bool tma, const BwdMaps& maps, const BwdParams& p, const Plan& pl, cudaStream_t st) {
  return tma ? bwd_dtype_v1<true, BwdMaps>(dtype, maps, p, pl, st)
             : bwd_dtype_v1<false, BwdMaps>(dtype, maps, p, pl, st);
}

// Sequence-sharded: the copy-engine path only (peer buffers are staged by TMA).
int v1_forward_sharded(int dtype, const ShardFwdMaps& maps, const FwdParams& p, const Plan& pl,
                       cudaStream_t st) {
  return fwd_dtype_v1<true, ShardFwdMaps>(dtype, maps, p, pl, st);
}

int v1_backward_sharded(int dtype, const ShardBwdMaps& maps, const BwdParams& p, const Plan& pl,
                        cudaStream_t st) {
  return bwd_dtype_v1<true, ShardBwdMaps>(dtype, maps, p, pl, st);
}

}  // namespace sbda
