// sbda_paths.cu -- SBDA attention over caller path tables: row i of batch b
// reads the sources index[b, i, 0..S-1] (S <= 4), as the reference's eager
// path does when a caller supplies path_indices/path_valid
// (BiAttn/left_v2.py:212-231 checks, 323-347 gather, 349-396 masked softmax).
//
//  * Forward: one row group of LPR lanes per row; each source's K/V row is
//    read straight from global memory (16-byte lane vectors).
//  * Backward, deterministic and atomic-free, in two passes:
//    - query pass: per row, p_s = exp(s_s - LSE) and dS_s = p_s (dO.v_s -
//      delta) scale for every source; writes dQ and the (p, dS) pairs to a
//      caller workspace [B, H, L, S, 2] (fp32);
//    - key pass: per key row j of a kv head, the (row, source) entries that
//      read j, from a caller-built inverse index (CSR per batch, entries in
//      a fixed order), summed over the query heads of the group:
//      dK_j = sum dS q_row, dV_j = sum p dO_row.
//  A source is used when its bit in source_mask[b, i] is set (path_valid,
//  causality, padding and segment rules are folded in by the caller).

#include "sbda_common.cuh"

namespace sbda {

struct PathParams {
  int B, H, Hkv, G, L, D, S;
  float scale;
  TensorArg q, k, v, out, dout, dq, dk, dv;
  const int32_t* index;     // [B, L, S]
  const uint8_t* mask;      // [B, L] source bits
  float* lse;               // [B, H, L]
  float* rec;               // [B, H, L, S, 2] (backward workspace)
  const int32_t* key_off;   // [B, L + 1]
  const int32_t* key_ent;   // [B, L * S]: i * S + s, grouped by key
};

template <typename TE>
__device__ __forceinline__ const TE* row_ptr(const TensorArg& t, int b, int h, int pos) {
  return reinterpret_cast<const TE*>(t.ptr) + (long long)b * t.sb + (long long)h * t.sh + (long long)pos * t.sl;
}

template <typename TE>
__device__ __forceinline__ Frag gather_row(const TensorArg& t, int b, int h, int pos, int D, int l, bool live) {
  const RowWords<TE> w = load_row_words<TE>(row_ptr<TE>(t, b, h, live ? pos : 0), D, l, live);
  return FragIO<TE>::from_words(w.w);
}

template <typename TE, int LPR>
__global__ void __launch_bounds__(kThreads) sbda_fwd_paths_kernel(const PathParams p) {
  constexpr int T = v2_tile(LPR);
  const int tid = threadIdx.x, grp = tid / LPR, l = tid % LPR;
  int bid = blockIdx.x;
  const int h = bid % p.H;
  bid /= p.H;
  const int nT = (p.L + T - 1) / T;
  const int t = bid % nT, b = bid / nT;
  const int hk = h / p.G;
  const float c1 = p.scale * kLog2e;
  float* lse = p.lse + ((long long)b * p.H + h) * p.L;
  TE* out = reinterpret_cast<TE*>(const_cast<void*>(p.out.ptr)) + (long long)b * p.out.sb + (long long)h * p.out.sh;
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    const int pos = t * T + grp * 4 + i;
    const bool inr = pos < p.L;  // uniform within a row group; every lane joins the shuffles
    const unsigned allow = inr ? p.mask[(long long)b * p.L + pos] : 0u;
    const Frag q = gather_row<TE>(p.q, b, h, pos, p.D, l, inr);
    float sc[4], m = -INFINITY;
    int src[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      sc[s] = -INFINITY;
      src[s] = 0;
      if (s < p.S) {
        const int j = ((allow >> s) & 1u) ? p.index[((long long)b * p.L + pos) * p.S + s] : -1;
        const bool use = (unsigned)j < (unsigned)p.L;  // an index outside [0, L) is not a source
        src[s] = use ? j : 0;
        const float a = lane_group_sum<LPR>(frag_dot(q, gather_row<TE>(p.k, b, hk, src[s], p.D, l, use)));
        if (use) sc[s] = a * c1;
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
      if (s < p.S && e[s] != 0.f) frag_axpy(o, e[s] * inv, gather_row<TE>(p.v, b, hk, src[s], p.D, l, true));
    if (inr) {
      store_frag<TE, true>(out + (long long)pos * p.out.sl, p.out.sd, p.D, l, o);
      if (l == 0) lse[pos] = any ? (m + __log2f(sum)) * kLn2 : -INFINITY;
    }
  }
}

template <typename TE, int LPR>
__global__ void __launch_bounds__(kThreads) sbda_bwd_paths_query_kernel(const PathParams p) {
  constexpr int T = v2_tile(LPR);
  const int tid = threadIdx.x, grp = tid / LPR, l = tid % LPR;
  int bid = blockIdx.x;
  const int h = bid % p.H;
  bid /= p.H;
  const int nT = (p.L + T - 1) / T;
  const int t = bid % nT, b = bid / nT;
  const int hk = h / p.G;
  const float c1 = p.scale * kLog2e;
  const float* lse = p.lse + ((long long)b * p.H + h) * p.L;
  TE* dq = reinterpret_cast<TE*>(const_cast<void*>(p.dq.ptr)) + (long long)b * p.dq.sb + (long long)h * p.dq.sh;
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    const int pos = t * T + grp * 4 + i;
    const bool inr = pos < p.L;
    const unsigned allow = inr ? p.mask[(long long)b * p.L + pos] : 0u;
    const float lq = inr ? lse[pos] * kLog2e : 0.f;
    const Frag q = gather_row<TE>(p.q, b, h, pos, p.D, l, inr);
    const Frag dO = gather_row<TE>(p.dout, b, h, pos, p.D, l, inr);
    float pr[4], bv[4], delta = 0.f;
    int src[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      pr[s] = bv[s] = 0.f;
      src[s] = 0;
      if (s < p.S) {
        const int j = ((allow >> s) & 1u) ? p.index[((long long)b * p.L + pos) * p.S + s] : -1;
        const bool use = (unsigned)j < (unsigned)p.L;
        src[s] = use ? j : 0;
        const float a = lane_group_sum<LPR>(frag_dot(q, gather_row<TE>(p.k, b, hk, src[s], p.D, l, use)));
        bv[s] = lane_group_sum<LPR>(frag_dot(dO, gather_row<TE>(p.v, b, hk, src[s], p.D, l, use)));
        if (use) pr[s] = fast_exp2(fmaf(a, c1, -lq));
        delta = fmaf(pr[s], bv[s], delta);
      }
    }
    Frag gq = frag_zero();
    float* rec = p.rec + (((long long)b * p.H + h) * p.L + (inr ? pos : 0)) * p.S * 2;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      if (s < p.S) {
        const float ds = pr[s] * (bv[s] - delta) * p.scale;
        if (ds != 0.f) frag_axpy(gq, ds, gather_row<TE>(p.k, b, hk, src[s], p.D, l, true));
        if (inr && l == 0) {
          rec[2 * s] = pr[s];
          rec[2 * s + 1] = ds;
        }
      }
    }
    if (inr) store_frag<TE, true>(dq + (long long)pos * p.dq.sl, p.dq.sd, p.D, l, gq);
  }
}

template <typename TE, int LPR>
__global__ void __launch_bounds__(kThreads) sbda_bwd_paths_key_kernel(const PathParams p) {
  constexpr int T = v2_tile(LPR);
  const int tid = threadIdx.x, grp = tid / LPR, l = tid % LPR;
  int bid = blockIdx.x;
  const int hk = bid % p.Hkv;
  bid /= p.Hkv;
  const int nT = (p.L + T - 1) / T;
  const int t = bid % nT, b = bid / nT;
  const int32_t* off = p.key_off + (long long)b * (p.L + 1);
  const int32_t* ent = p.key_ent + (long long)b * p.L * p.S;
  TE* dk = reinterpret_cast<TE*>(const_cast<void*>(p.dk.ptr)) + (long long)b * p.dk.sb + (long long)hk * p.dk.sh;
  TE* dv = reinterpret_cast<TE*>(const_cast<void*>(p.dv.ptr)) + (long long)b * p.dv.sb + (long long)hk * p.dv.sh;
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    const int j = t * T + grp * 4 + i;
    if (j >= p.L) break;  // the rest of this group's keys are past L too; no shuffles below
    Frag ak = frag_zero(), av = frag_zero();
    const int n_ent = p.L * p.S;
    const int e_end = min(off[j + 1], n_ent);
#pragma unroll 1
    for (int e = max(off[j], 0); e < e_end; ++e) {
      const int code = ent[e];
      if ((unsigned)code >= (unsigned)n_ent) continue;  // malformed entry: skipped
      const int row = code / p.S, s = code - row * p.S;
#pragma unroll 1
      for (int gi = 0; gi < p.G; ++gi) {
        const int h = hk * p.G + gi;
        const float* rec = p.rec + (((long long)b * p.H + h) * p.L + row) * p.S * 2 + 2 * s;
        const float pr = rec[0], ds = rec[1];
        if (pr == 0.f && ds == 0.f) continue;
        frag_axpy(ak, ds, gather_row<TE>(p.q, b, h, row, p.D, l, true));
        frag_axpy(av, pr, gather_row<TE>(p.dout, b, h, row, p.D, l, true));
      }
    }
    store_frag<TE, true>(dk + (long long)j * p.dk.sl, p.dk.sd, p.D, l, ak);
    store_frag<TE, true>(dv + (long long)j * p.dv.sl, p.dv.sd, p.D, l, av);
  }
}

namespace {

template <typename TE, int LPR>
int launch_paths(int which, const PathParams& p, cudaStream_t st) {
  constexpr int T = v2_tile(LPR);
  const long long nT = (p.L + T - 1) / T;
  if (which == 0) {
    sbda_fwd_paths_kernel<TE, LPR><<<(unsigned)(p.B * p.H * nT), kThreads, 0, st>>>(p);
  } else {
    sbda_bwd_paths_query_kernel<TE, LPR><<<(unsigned)(p.B * p.H * nT), kThreads, 0, st>>>(p);
    if (cudaGetLastError() != cudaSuccess) return SBDA_ERR_CUDA;
    sbda_bwd_paths_key_kernel<TE, LPR><<<(unsigned)(p.B * p.Hkv * nT), kThreads, 0, st>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? SBDA_OK : SBDA_ERR_CUDA;
}

template <typename TE>
int paths_lpr(int which, int lpr, const PathParams& p, cudaStream_t st) {
  if constexpr (sizeof(TE) == 4) {
    if (lpr == 4) return launch_paths<TE, 4>(which, p, st);
  }
  if (lpr == 8) return launch_paths<TE, 8>(which, p, st);
  if (lpr == 16) return launch_paths<TE, 16>(which, p, st);
  return SBDA_ERR_UNSUPPORTED;
}

int paths_dispatch(int dtype, int which, int lpr, const PathParams& p, cudaStream_t st) {
  if (dtype == SBDA_DTYPE_F32) return paths_lpr<float>(which, lpr, p, st);
  if (dtype == SBDA_DTYPE_F16) return paths_lpr<__half>(which, lpr, p, st);
  return paths_lpr<__nv_bfloat16>(which, lpr, p, st);
}

TensorArg targ(const sbda_tensor& t) {
  TensorArg a;
  a.ptr = t.data;
  a.sb = t.stride_b;
  a.sh = t.stride_h;
  a.sl = t.stride_l;
  a.sd = t.stride_d;
  return a;
}

// Shapes, dtypes and the vector-layout rule (16-byte aligned rows with unit
// channel stride: rows are read as 16-byte lane vectors).  Returns a status;
// on success *lpr is the lanes per row.
int paths_check(int dtype, const sbda_shape& s, int n_sources, std::initializer_list<const sbda_tensor*> ts,
                std::initializer_list<int64_t> heads, int* lpr) {
  if (dtype != SBDA_DTYPE_F32 && dtype != SBDA_DTYPE_F16 && dtype != SBDA_DTYPE_BF16) return SBDA_ERR_DTYPE;
  if (s.batch < 0 || s.heads < 0 || s.kv_heads < 0 || s.length < 0 || s.head_dim < 1 || s.head_dim > 128)
    return SBDA_ERR_INVALID;
  if (s.kv_heads == 0 ? s.heads != 0 : s.heads % s.kv_heads) return SBDA_ERR_INVALID;
  if (n_sources < 1 || n_sources > 4) return SBDA_ERR_INVALID;
  if (s.length > ((int64_t)1 << 30) / 4 || s.batch * s.heads > ((int64_t)1 << 31) / 2) return SBDA_ERR_UNSUPPORTED;
  const int e = dtype == SBDA_DTYPE_F32 ? 4 : 2;
  if ((s.head_dim * e) % 16) return SBDA_ERR_UNSUPPORTED;
  auto h = heads.begin();
  for (const sbda_tensor* t : ts) {
    if (!t->data || reinterpret_cast<uintptr_t>(t->data) % 16) return SBDA_ERR_INVALID;
    if (s.head_dim > 1 && t->stride_d != 1) return SBDA_ERR_UNSUPPORTED;
    const int64_t sizes[3] = {s.batch, *h, s.length};
    const int64_t strides[3] = {t->stride_b, t->stride_h, t->stride_l};
    for (int i = 0; i < 3; ++i)
      if (sizes[i] > 1 && (strides[i] <= 0 || (strides[i] * e) % 16)) return SBDA_ERR_UNSUPPORTED;
    ++h;
  }
  int pitch = 128;
  while (pitch < s.head_dim * e) pitch *= 2;
  *lpr = pitch / (e == 4 ? 32 : 16);
  if (*lpr != 4 && *lpr != 8 && *lpr != 16) return SBDA_ERR_UNSUPPORTED;
  return SBDA_OK;
}

void paths_params(PathParams* p, const sbda_shape& s, int n_sources, float scale) {
  memset(p, 0, sizeof(*p));
  p->B = (int)s.batch;
  p->H = (int)s.heads;
  p->Hkv = (int)s.kv_heads;
  p->G = (int)(s.heads / s.kv_heads);
  p->L = (int)s.length;
  p->D = (int)s.head_dim;
  p->S = n_sources;
  p->scale = scale;
}

}  // namespace
}  // namespace sbda

using namespace sbda;

extern "C" int sbda_b200_forward_paths(int dtype, sbda_shape shape, int32_t n_sources, float scale,
                                       sbda_tensor q, sbda_tensor k, sbda_tensor v, const int32_t* path_index,
                                       const uint8_t* source_mask, sbda_tensor out, float* lse, void* stream) {
  int lpr = 0;
  if (shape.batch == 0 || shape.heads == 0 || shape.length == 0) {
    const int st = paths_check(dtype, shape, n_sources, {}, {}, &lpr);
    return st == SBDA_ERR_UNSUPPORTED ? SBDA_OK : st;
  }
  int st = paths_check(dtype, shape, n_sources, {&q, &k, &v, &out},
                       {shape.heads, shape.kv_heads, shape.kv_heads, shape.heads}, &lpr);
  if (st != SBDA_OK) return st;
  if (!path_index || !source_mask || !lse) return SBDA_ERR_INVALID;
  PathParams p;
  paths_params(&p, shape, n_sources, scale);
  p.q = targ(q);
  p.k = targ(k);
  p.v = targ(v);
  p.out = targ(out);
  p.index = path_index;
  p.mask = source_mask;
  p.lse = lse;
  return paths_dispatch(dtype, 0, lpr, p, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int64_t sbda_b200_paths_workspace_floats(sbda_shape shape, int32_t n_sources) {
  if (shape.batch < 0 || shape.heads < 0 || shape.length < 0 || n_sources < 1) return 0;
  return shape.batch * shape.heads * shape.length * (int64_t)n_sources * 2;
}

extern "C" int sbda_b200_backward_paths(int dtype, sbda_shape shape, int32_t n_sources, float scale,
                                        sbda_tensor q, sbda_tensor k, sbda_tensor v, const int32_t* path_index,
                                        const uint8_t* source_mask, const int32_t* key_offsets,
                                        const int32_t* key_entries, sbda_tensor grad_out, const float* lse,
                                        float* workspace, int64_t workspace_floats, sbda_tensor grad_q,
                                        sbda_tensor grad_k, sbda_tensor grad_v, void* stream) {
  int lpr = 0;
  if (shape.batch == 0 || shape.heads == 0 || shape.length == 0) {
    const int st = paths_check(dtype, shape, n_sources, {}, {}, &lpr);
    return st == SBDA_ERR_UNSUPPORTED ? SBDA_OK : st;
  }
  int st = paths_check(dtype, shape, n_sources, {&q, &k, &v, &grad_out, &grad_q, &grad_k, &grad_v},
                       {shape.heads, shape.kv_heads, shape.kv_heads, shape.heads, shape.heads, shape.kv_heads,
                        shape.kv_heads},
                       &lpr);
  if (st != SBDA_OK) return st;
  if (!path_index || !source_mask || !key_offsets || !key_entries || !lse || !workspace) return SBDA_ERR_INVALID;
  if (workspace_floats < sbda_b200_paths_workspace_floats(shape, n_sources)) return SBDA_ERR_INVALID;
  PathParams p;
  paths_params(&p, shape, n_sources, scale);
  p.q = targ(q);
  p.k = targ(k);
  p.v = targ(v);
  p.dout = targ(grad_out);
  p.dq = targ(grad_q);
  p.dk = targ(grad_k);
  p.dv = targ(grad_v);
  p.index = path_index;
  p.mask = source_mask;
  p.lse = const_cast<float*>(lse);
  p.rec = workspace;
  p.key_off = key_offsets;
  p.key_ent = key_entries;
  return paths_dispatch(dtype, 1, lpr, p, reinterpret_cast<cudaStream_t>(stream));
}
