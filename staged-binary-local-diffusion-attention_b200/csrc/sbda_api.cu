// sbda_api.cu -- host side of the C ABI (include/sbda_b200.h): argument
// validation, tile planning, tensor-map encoding and kernel selection.

#include "sbda_common.cuh"

#include <atomic>
#include <map>
#include <mutex>
#include <string.h>
#include <tuple>

namespace sbda {

__device__ unsigned int g_device_status = 0;

// Device address of g_device_status per device (kernels receive it as a
// pointer so every translation unit reports into one word).
unsigned* status_ptr() {
  static std::atomic<unsigned*> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return nullptr;
  if (dev < 64) {
    unsigned* p = cache[dev].load(std::memory_order_acquire);
    if (p) return p;
  }
  void* addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_device_status) != cudaSuccess) return nullptr;
  if (dev < 64) cache[dev].store(static_cast<unsigned*>(addr), std::memory_order_release);
  return static_cast<unsigned*>(addr);
}

// Kernel families a call may be pinned to (the *_ex entry points): 0 = automatic,
// 1 = general kernels, 2 = uniform kernels.  There is no process-wide setting.
constexpr int kFamilyAuto = 0, kFamilyGeneral = 1, kFamilyUniform = 2;
bool family_ok(int family) { return family >= kFamilyAuto && family <= kFamilyUniform; }

// SM count of the current device, read once per device.
int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return n;
  if (dev >= 0 && dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

// The tensor-map encoder is a driver call and needs a current context on the
// calling thread.  A thread that has only run cached runtime calls (autograd's
// worker thread on its first backward, for instance) may have none yet: bind
// the current device's primary context, so the caller can retry the encode.
bool bind_current_context() {
  int dev = 0;
  return cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess;
}

int elem_size(int dtype) { return dtype == SBDA_DTYPE_F32 ? 4 : 2; }

CUtensorMapDataType map_dtype(int dtype) {
  return dtype == SBDA_DTYPE_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
         : dtype == SBDA_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// Row pitch of a staged tile: D padded to a power of two, at least 128 bytes.
int row_pitch(int64_t D, int e) {
  int p = 128;
  while (p < D * e) p *= 2;
  return p;
}

struct View {
  const void* ptr;
  int64_t heads;
  sbda_tensor t;
};

// A view can be staged by the copy engine / written with 16-byte vectors when
// its base and the byte strides of every non-trivial outer dimension are
// multiples of 16 and channels are contiguous.
bool vector_ok(const sbda_tensor& t, int64_t B, int64_t H, int64_t L, int64_t D, int e) {
  if (reinterpret_cast<uintptr_t>(t.data) % 16) return false;
  if (D > 1 && t.stride_d != 1) return false;
  if ((D * e) % 16) return false;
  const int64_t sizes[3] = {B, H, L};
  const int64_t strides[3] = {t.stride_b, t.stride_h, t.stride_l};
  for (int i = 0; i < 3; ++i)
    if (sizes[i] > 1 && (strides[i] <= 0 || (strides[i] * e) % 16)) return false;
  return true;
}

// Encodes the (D, outer...) 4-D map of a view with a box of `rows` positions.
// Outer dimensions are ordered by increasing stride; `slots` records where
// position / head / batch land (2 bits each).
bool encode_map(CUtensorMap* map, unsigned* slots, const sbda_tensor& t, int dtype, int64_t B, int64_t H,
                int64_t L, int64_t D, int pitch, int rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const int e = elem_size(dtype);
  int64_t size[3] = {L, H, B};
  int64_t stride[3] = {t.stride_l * e, t.stride_h * e, t.stride_b * e};
  int64_t big = 16;
  for (int i = 0; i < 3; ++i)
    if (size[i] > 1) big = (stride[i] * size[i] > big) ? stride[i] * size[i] : big;
  for (int i = 0; i < 3; ++i)
    if (size[i] <= 1) stride[i] = ((big + 15) / 16) * 16;  // trivial dims go outermost
  int order[3] = {0, 1, 2};
  for (int a = 0; a < 3; ++a)
    for (int c = a + 1; c < 3; ++c)
      if (stride[order[c]] < stride[order[a]]) {
        const int tmp = order[a];
        order[a] = order[c];
        order[c] = tmp;
      }
  cuuint64_t gdim[4] = {(cuuint64_t)D, 0, 0, 0};
  cuuint64_t gstride[3];
  cuuint32_t box[4] = {(cuuint32_t)(pitch / e), 1, 1, 1};
  cuuint32_t estride[4] = {1, 1, 1, 1};
  unsigned s = 0;
  for (int k = 0; k < 3; ++k) {
    const int d = order[k];
    gdim[k + 1] = (cuuint64_t)size[d];
    gstride[k] = (cuuint64_t)stride[d];
    if (d == 0) {
      box[k + 1] = (cuuint32_t)rows;
      s |= (unsigned)(k + 1);
    } else if (d == 1) {
      s |= (unsigned)(k + 1) << 2;
    } else {
      s |= (unsigned)(k + 1) << 4;
    }
  }
  *slots = s;
  auto encode = [&] {
    return enc(map, map_dtype(dtype), 4, const_cast<void*>(t.data), gdim, gstride, box, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r != CUDA_SUCCESS && bind_current_context()) r = encode();
  return r == CUDA_SUCCESS;
}

// 2-D map over the fp32 log-sum-exp rows [rows, L] (contiguous); needs the
// row stride L * 4 to be a multiple of 16 bytes.
bool encode_lse_map(CUtensorMap* map, const float* lse, int64_t rows, int64_t L, int box) {
  auto enc = encode_fn();
  if (!enc || L % 4 || reinterpret_cast<uintptr_t>(lse) % 16) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)L, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)(L * 4)};
  cuuint32_t boxd[2] = {(cuuint32_t)box, 1};
  cuuint32_t estride[2] = {1, 1};
  auto encode = [&] {
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(lse), gdim, gstride, boxd, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r != CUDA_SUCCESS && bind_current_context()) r = encode();
  return r == CUDA_SUCCESS;
}

// Splits offsets into the near window and at most one far offset for a tile
// height, and sizes the staged regions.  Returns false when the offsets need
// two far tiles at this tile height.
bool plan_for_tile(const int32_t* off, int n, int64_t L, int tile, int pitch, Plan* pl) {
  Geometry g;
  memset(&g, 0, sizeof(g));
  g.S = n;
  int nfar = 0;
  for (int s = 0; s < n; ++s) {
    g.off[s] = off[s];
    if (off[s] > tile) {
      g.is_far[s] = 1;
      g.f = off[s];
      ++nfar;
    } else if (off[s] > g.Hn) {
      g.Hn = off[s];
    }
  }
  if (nfar > 1) return false;
  g.has_far = nfar;
  g.nT = (int)((L + tile - 1) / tile);
  g.R = g.A = g.rem = 0;
  if (g.has_far && g.f % tile == 0) {
    const int R = g.f / tile;
    if (R < g.nT) {
      g.R = R;
      g.A = (g.nT + R - 1) / R;
      g.rem = g.nT - (g.A - 1) * R;
    }
  }
  const size_t P = pitch;
  const size_t T = tile, Hn = g.Hn, F = g.has_far;
  pl->tile = tile;
  pl->pitch = pitch;
  pl->nv = pitch / 128;
  pl->g = g;
  pl->smem_fwd = (T + 2 * (Hn + T) + 2 * T * F) * P + 16;
  const size_t nc = T + Hn + F * T;
  pl->smem_bwd = (2 * (T + Hn) + 2 * (T + 2 * Hn) + F * (2 * (T + Hn) + 2 * T + 2 * (Hn + T))) * P +
                 nc * 4 * sizeof(float2) + 16;
  return true;
}

constexpr size_t kMaxSmem = 227 * 1024;

int make_plan(const int32_t* off, int n, int64_t L, int64_t D, int e, Plan* pl) {
  const int pitch = row_pitch(D, e);
  const int nv = pitch / 128;
  const int elems = nv * (16 / e);  // floats per lane per row
  // Tile heights instantiated per pitch, largest first.  The backward keeps
  // TILE/16 * EPL * 2 fp32 key accumulators per thread; keep that <= 64.
  int tiles[2] = {64, 0};
  if (nv == 2) {
    tiles[0] = elems <= 8 ? 64 : 32;
    tiles[1] = elems <= 8 ? 32 : 0;
  } else if (nv == 4) {
    tiles[0] = 32;
    tiles[1] = 16;
  }
  for (int i = 0; i < 2 && tiles[i]; ++i) {
    Plan cand;
    if (!plan_for_tile(off, n, L, tiles[i], pitch, &cand)) continue;
    if (cand.smem_fwd > kMaxSmem || cand.smem_bwd > kMaxSmem) continue;
    *pl = cand;
    return SBDA_OK;
  }
  return SBDA_ERR_UNSUPPORTED;
}


// Plan of the windowed kernels (sbda_v2.cu).  They serve MHA schedules whose
// near offsets lie in {0, 1, 2} with at most one far offset d > 2; the
// backward walks chains when d is a multiple of the tile height.
// K/V rows the forward stages before its tile: the far offset when it is shorter
// than a tile (its sources then share the window), else the 2 rows of offsets 1, 2.
int fwd_window_lead(const V2Geometry& g, int T) { return g.has_far && g.d < T ? g.d : 2; }

// LSE rows staged per backward step: the Q/dO slot height rounded up to 32
// (fp32 rows; 128-byte multiples).
int lse_box_rows(const V2Geometry& g, int T) { return (T + g.halo + 31) / 32 * 32; }

// Dynamic shared memory of the windowed backward for a geometry: K/V slots,
// two Q/dO slots, the softmax-record ring, two LSE slots and the barriers.
size_t bwd_smem(const V2Geometry& g, int T, int pitch) {
  const size_t P = pitch, Tz = T, hz = g.halo;
  const size_t nkv = g.mode == 0 ? 2 : 1, kvr = g.mode == 2 ? Tz + g.d : Tz + 2 * hz, qdr = Tz + hz;
  return nkv * 2 * kvr * P + 2 * 2 * qdr * P + v2_ring_floats(T) * sizeof(float) + 128 +
         2 * (size_t)lse_box_rows(g, T) * 4 + 16;
}

// Largest per-CTA dynamic shared memory that still lets three CTAs share an
// SM (228 KB per SM, 1 KB reserved per CTA).
constexpr size_t kSmemThreeCtas = 228 * 1024 / 3 - 1024;

// Segment length for `chains` walks of `len` tiles each on `slots` resident
// CTAs.  Among splits that give at least 3.5 waves of CTAs (so the block
// scheduler can even out CTAs that run long), minimise (waves, rounded up) x
// (steps per CTA); a segment that is not the top of its walk first runs a
// carry-only tile when `pre` is set, so segments are at least four tiles then.
// Problems too small for 3.5 waves take the split with the most CTAs.
int balanced_segment(int64_t chains, int len, bool pre, int64_t slots) {
  int best = len;
  bool best_full = false;
  int64_t best_cost = 0, best_ctas = 0;
  for (int segs = 1; segs <= len && segs <= 8192; ++segs) {
    const int seg = (len + segs - 1) / segs;
    if (pre && seg < 4 && segs > 1) break;
    const int n_seg = (len + seg - 1) / seg;
    if (n_seg != segs) continue;  // same split as a smaller count
    const int64_t ctas = chains * n_seg;
    const bool full = 2 * ctas >= 7 * slots;
    const int64_t cost = (ctas + slots - 1) / slots * (seg + (pre && n_seg > 1 ? 1 : 0));
    const bool better = full ? (!best_full || cost < best_cost) : (!best_full && ctas > best_ctas);
    if (segs == 1 || better) {
      best = seg;
      best_full = full;
      best_cost = cost;
      best_ctas = ctas;
    }
  }
  return best;
}

// balanced_segment searches up to 8192 splits; a layer calls it with the same
// arguments every step, so results are kept (a few hundred entries at most).
int balanced_segment_cached(int64_t chains, int len, bool pre, int64_t slots) {
  static std::mutex mu;
  static std::map<std::tuple<int64_t, int, bool, int64_t>, int> cache;
  const auto key = std::make_tuple(chains, len, pre, slots);
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int seg = balanced_segment(chains, len, pre, slots);
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 512) cache.clear();
  cache.emplace(key, seg);
  return seg;
}

// L: rows of this call (a shard when sequence-sharded); total_L: positions of
// the whole sequence (offsets at or beyond it never have a source).
bool plan_v2(const int32_t* off, int n, int64_t L, int64_t D, int e, int64_t G, int64_t B, int64_t H,
             V2Plan* pl, int64_t total_L = -1) {
  if (total_L < 0) total_L = L;
  if (G != 1) return false;
  const int pitch = row_pitch(D, e);
  const int lane_bytes = e == 4 ? 32 : 16;
  const int lpr = pitch / lane_bytes;
  if (lpr != 4 && lpr != 8 && lpr != 16) return false;
  const int T = v2_tile(lpr);
  V2Geometry g;
  memset(&g, 0, sizeof(g));
  int nfar = 0;
  for (int s = 0; s < n; ++s) {
    if (off[s] == 0) g.has0 = 1;
    else if (off[s] == 1) g.has1 = 1;
    else if (off[s] == 2) g.has2 = 1;
    else if (off[s] < total_L) {
      g.d = off[s];
      ++nfar;
    }
    // a far offset >= total_L never has a valid source: it drops out of every row
  }
  if (nfar > 1) return false;
  g.has_far = nfar;
  g.nT = (int)((L + T - 1) / T);
  if (g.has_far && g.d % T == 0) {
    // Chains t, t + R, ... of this call's tiles; a shard shorter than d holds
    // one tile of each of its nT chains.
    g.R = g.d / T;
    g.chains = g.R < g.nT ? g.R : g.nT;
    g.A = (g.nT + g.R - 1) / g.R;
    g.rem = g.nT - (g.A - 1) * g.R;
  }
  if (g.has_far && g.d >= T) {
    if (g.d % T) return false;
    g.mode = 0;
    g.halo = 2;
  } else {
    g.mode = 1;
    g.halo = g.has_far ? (g.d > 2 ? g.d : 2) : 2;
    // Local mode stages T + 2d K/V rows and T + d Q/dO rows.  When that keeps
    // fewer than three CTAs on an SM, the local carry walk (T + d and T + 2
    // rows) serves d % 4 == 0 instead.
    if (g.has_far && g.d % 4 == 0 && bwd_smem(g, T, pitch) > kSmemThreeCtas) {
      g.mode = 2;
      g.halo = 2;
    }
  }
  pl->lpr = lpr;
  pl->tile = T;
  pl->pitch = pitch;
  // Forward: [Q] + K/V rows [i0 - lead, i0 + T) (lead = d for a far offset under a
  // tile, else 2) + a separate far tile for longer far offsets.
  const int fwd_lead = fwd_window_lead(g, T);
  pl->smem_fwd = (size_t)(T + 2 * (T + fwd_lead) + (g.has_far && g.d >= T ? 2 * T : 0)) * pitch + 16;
  pl->lse_box = lse_box_rows(g, T);
  pl->smem_bwd = bwd_smem(g, T, pitch);
  if (pl->smem_fwd > kMaxSmem || pl->smem_bwd > kMaxSmem) return false;
  // Backward work split: walks of `chains` x `len` tiles cut into segments,
  // one CTA each.
  const int64_t chains = g.mode == 0 ? B * H * (int64_t)g.chains : B * H;
  const int len = g.mode == 0 ? g.A : g.nT;
  g.seg = balanced_segment_cached(chains, len, g.mode != 1, (int64_t)sm_count() * 3);
  g.segs = (len + g.seg - 1) / g.seg;
  pl->blocks_bwd = (unsigned)(chains * g.segs);
  pl->g = g;
  return true;
}

// Plan of the uniform kernels (sbda_v3.cu): any offsets, each source its own
// staged tile.  Tile height as in the windowed kernels (four rows per row group).
bool plan_v3(int64_t D, int e, V3Plan* pl) {
  const int pitch = row_pitch(D, e);
  const int lane_bytes = e == 4 ? 32 : 16;
  const int lpr = pitch / lane_bytes;
  if (lpr != 4 && lpr != 8 && lpr != 16) return false;
  if (lpr == 4 && e != 4) return false;
  const size_t tile_bytes = (size_t)v2_tile(lpr) * pitch;
  pl->lpr = lpr;
  pl->tile = v2_tile(lpr);
  pl->pitch = pitch;
  pl->smem_fwd = (1 + 2 * 4) * tile_bytes + 16;  // sized for four sources
  pl->smem_bwd = (2 + 2 * 4) * tile_bytes + 16;
  return pl->smem_fwd <= kMaxSmem && pl->smem_bwd <= kMaxSmem;
}

void v3_params(V3Params* p, const sbda_shape& shape, const int32_t* off, int n, float scale, int tile) {
  memset(p, 0, sizeof(*p));
  p->B = (int)shape.batch;
  p->H = (int)shape.heads;
  p->Hkv = (int)shape.kv_heads;
  p->G = (int)(shape.heads / shape.kv_heads);
  p->L = (int)shape.length;
  p->D = (int)shape.head_dim;
  p->scale = scale;
  p->S = n;
  p->nT = (int)((shape.length + tile - 1) / tile);
  p->o_min = off[0];
  for (int s = 0; s < n; ++s) {
    p->off[s] = off[s];
    if (off[s] < p->o_min) {
      p->o_min = off[s];
      p->s_q = s;
    }
  }
  p->status = status_ptr();
}

int validate(int dtype, const sbda_shape& s, const int32_t* off, int n) {
  if (dtype != SBDA_DTYPE_F32 && dtype != SBDA_DTYPE_F16 && dtype != SBDA_DTYPE_BF16) return SBDA_ERR_DTYPE;
  if (s.batch < 0 || s.heads < 0 || s.kv_heads < 0 || s.length < 0 || s.head_dim < 1) return SBDA_ERR_INVALID;
  if (s.head_dim > 128) return SBDA_ERR_INVALID;
  if (s.kv_heads == 0 ? s.heads != 0 : s.heads % s.kv_heads) return SBDA_ERR_INVALID;
  if (s.length > (int64_t)1 << 30 || s.batch * s.heads > ((int64_t)1 << 31) / 2) return SBDA_ERR_UNSUPPORTED;
  if (!off || n < 1 || n > 4) return SBDA_ERR_INVALID;
  for (int a = 0; a < n; ++a) {
    if (off[a] < 0) return SBDA_ERR_INVALID;
    for (int c = a + 1; c < n; ++c)
      if (off[a] == off[c]) return SBDA_ERR_INVALID;
  }
  return SBDA_OK;
}

TensorArg arg_of(const sbda_tensor& t) {
  return TensorArg{t.data, t.stride_b, t.stride_h, t.stride_l, t.stride_d};
}

// The whole sequence on one GPU.
ShardInfo single_shard(int64_t L, const float* lse) {
  ShardInfo s;
  memset(&s, 0, sizeof(s));
  s.rank = 0;
  s.world = 1;
  s.shard_len = (int)L;
  s.pos0 = 0;
  s.total_len = (int)L;
  s.lse[0] = lse;
  return s;
}


// Shape/stride eligibility shared by forward and backward.
bool tensors_vector_ok(std::initializer_list<const sbda_tensor*> ts, int64_t B, int64_t L, int64_t D, int e,
                       std::initializer_list<int64_t> heads) {
  auto h = heads.begin();
  for (const sbda_tensor* t : ts) {
    if (!vector_ok(*t, B, *h, L, D, e)) return false;
    ++h;
  }
  return true;
}

// Uniform-kernel calls (also the masked entry points).  Shapes and pointers
// are validated by the caller; `vec` says whether every view suits TMA.
int uniform_forward(int dtype, const sbda_shape& shape, const int32_t* offsets, int n, float scale,
                    const sbda_tensor& q, const sbda_tensor& k, const sbda_tensor& v, const uint8_t* mask,
                    const sbda_tensor& out, float* lse, bool vec, cudaStream_t stream) {
  const int e = elem_size(dtype);
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, L = shape.length, D = shape.head_dim;
  V3Plan p3;
  if (!plan_v3(D, e, &p3)) return SBDA_ERR_UNSUPPORTED;
  V3Params p;
  v3_params(&p, shape, offsets, n, scale, p3.tile);
  p.q = arg_of(q);
  p.k = arg_of(k);
  p.v = arg_of(v);
  p.out = arg_of(out);
  p.lse = lse;
  p.mask = mask;
  FwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  const bool tma = vec && encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, L, D, p3.pitch, p3.tile) &&
                   encode_map(&maps.kT, &p.slots_k, k, dtype, B, Hkv, L, D, p3.pitch, p3.tile) &&
                   encode_map(&maps.vT, &p.slots_v, v, dtype, B, Hkv, L, D, p3.pitch, p3.tile);
  return v3_forward(dtype, tma, maps, p, p3, stream);
}

int uniform_backward(int dtype, const sbda_shape& shape, const int32_t* offsets, int n, float scale,
                     const sbda_tensor& q, const sbda_tensor& k, const sbda_tensor& v, const uint8_t* mask,
                     const sbda_tensor& grad_out, const float* lse, const sbda_tensor& grad_q,
                     const sbda_tensor& grad_k, const sbda_tensor& grad_v, bool vec, cudaStream_t stream) {
  const int e = elem_size(dtype);
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, L = shape.length, D = shape.head_dim;
  V3Plan p3;
  if (!plan_v3(D, e, &p3)) return SBDA_ERR_UNSUPPORTED;
  V3Params p;
  v3_params(&p, shape, offsets, n, scale, p3.tile);
  p.q = arg_of(q);
  p.k = arg_of(k);
  p.v = arg_of(v);
  p.dout = arg_of(grad_out);
  p.dq = arg_of(grad_q);
  p.dk = arg_of(grad_k);
  p.dv = arg_of(grad_v);
  p.lse = const_cast<float*>(lse);
  p.mask = mask;
  BwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  const bool tma = vec && encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, L, D, p3.pitch, p3.tile) &&
                   encode_map(&maps.dT, &p.slots_d, grad_out, dtype, B, H, L, D, p3.pitch, p3.tile) &&
                   encode_map(&maps.kT, &p.slots_k, k, dtype, B, Hkv, L, D, p3.pitch, p3.tile) &&
                   encode_map(&maps.vT, &p.slots_v, v, dtype, B, Hkv, L, D, p3.pitch, p3.tile);
  return v3_backward(dtype, tma, maps, p, p3, stream);
}

}  // namespace sbda

using namespace sbda;

extern "C" int sbda_b200_abi_version(void) { return SBDA_B200_ABI_VERSION; }

extern "C" const char* sbda_b200_status_string(int status) {
  switch (status) {
    case SBDA_OK: return "ok";
    case SBDA_ERR_INVALID: return "invalid argument (shape, stride, offsets or pointer)";
    case SBDA_ERR_DTYPE: return "unsupported SBDA dtype";
    case SBDA_ERR_UNSUPPORTED: return "offsets or shape outside the kernel envelope";
    case SBDA_ERR_CUDA: return "CUDA runtime error";
    case SBDA_ERR_DEVICE: return "device-side fault reported by an SBDA kernel";
    default: return "unknown SBDA status";
  }
}

extern "C" int sbda_b200_forward_ex(int family, int dtype, sbda_shape shape, const int32_t* offsets,
                                    int32_t n_offsets, float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                                    sbda_tensor out, float* lse, void* stream) {
  if (!family_ok(family)) return SBDA_ERR_INVALID;
  int st = validate(dtype, shape, offsets, n_offsets);
  if (st != SBDA_OK) return st;
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, L = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || L == 0) return SBDA_OK;
  if (!q.data || !k.data || !v.data || !out.data || !lse) return SBDA_ERR_INVALID;
  const int e = elem_size(dtype);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = tensors_vector_ok({&q, &k, &v, &out}, B, L, D, e, {H, Hkv, Hkv, H});

  V2Plan p2;
  // The windowed forward serves grouped-query attention too (K/V rows from kv head h / G); its
  // plan does not depend on G, so it is made as for MHA.
  if (family == kFamilyAuto && plan_v2(offsets, n_offsets, L, D, e, 1, B, H, &p2)) {
    FwdV2Params p;
    memset(&p, 0, sizeof(p));
    p.G = (int)(H / Hkv);
    p.B = (int)B;
    p.H = (int)H;
    p.L = (int)L;
    p.D = (int)D;
    p.scale = scale;
    p.g = p2.g;
    p.q = arg_of(q);
    p.k = arg_of(k);
    p.v = arg_of(v);
    p.out = arg_of(out);
    p.lse = lse;
    p.status = status_ptr();
    p.sh = single_shard(L, lse);
    FwdMaps maps;
    memset(&maps, 0, sizeof(maps));
    bool tma = vec;
    if (tma) {
      unsigned dummy;
      tma = encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, L, D, p2.pitch, p2.tile) &&
            encode_map(&maps.kT, &p.slots_k, k, dtype, B, Hkv, L, D, p2.pitch, p2.tile) &&
            encode_map(&maps.vT, &p.slots_v, v, dtype, B, Hkv, L, D, p2.pitch, p2.tile) &&
            encode_map(&maps.kH, &dummy, k, dtype, B, Hkv, L, D, p2.pitch, fwd_window_lead(p2.g, p2.tile)) &&
            encode_map(&maps.vH, &dummy, v, dtype, B, Hkv, L, D, p2.pitch, fwd_window_lead(p2.g, p2.tile));
    }
    return v2_forward(dtype, tma, maps, p, p2, s);
  }

  Plan pl;
  st = family == kFamilyUniform ? SBDA_ERR_UNSUPPORTED : make_plan(offsets, n_offsets, L, D, e, &pl);
  if (st == SBDA_ERR_UNSUPPORTED)  // several far offsets (or forced): the uniform kernels
    return uniform_forward(dtype, shape, offsets, n_offsets, scale, q, k, v, nullptr, out, lse, vec, s);
  if (st != SBDA_OK) return st;
  FwdParams p;
  memset(&p, 0, sizeof(p));
  p.B = (int)B;
  p.H = (int)H;
  p.Hkv = (int)Hkv;
  p.G = (int)(H / Hkv);
  p.L = (int)L;
  p.D = (int)D;
  p.scale = scale;
  p.g = pl.g;
  p.q = arg_of(q);
  p.k = arg_of(k);
  p.v = arg_of(v);
  p.out = arg_of(out);
  p.lse = lse;
  p.status = status_ptr();
  p.sh = single_shard(L, lse);
  FwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  bool tma = vec;
  if (tma) {
    unsigned dummy;
    tma = encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.kT, &p.slots_k, k, dtype, B, Hkv, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.vT, &p.slots_v, v, dtype, B, Hkv, L, D, pl.pitch, pl.tile);
    if (tma && pl.g.Hn > 0)
      tma = encode_map(&maps.kH, &dummy, k, dtype, B, Hkv, L, D, pl.pitch, pl.g.Hn) &&
            encode_map(&maps.vH, &dummy, v, dtype, B, Hkv, L, D, pl.pitch, pl.g.Hn);
  }
  return v1_forward(dtype, tma, maps, p, pl, s);
}

extern "C" int sbda_b200_forward(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                 float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v, sbda_tensor out,
                                 float* lse, void* stream) {
  return sbda_b200_forward_ex(kFamilyAuto, dtype, shape, offsets, n_offsets, scale, q, k, v, out, lse, stream);
}

extern "C" int sbda_b200_backward_ex(int family, int dtype, sbda_shape shape, const int32_t* offsets,
                                     int32_t n_offsets, float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                                     sbda_tensor grad_out, const float* lse, sbda_tensor grad_q,
                                     sbda_tensor grad_k, sbda_tensor grad_v, void* stream) {
  if (!family_ok(family)) return SBDA_ERR_INVALID;
  int st = validate(dtype, shape, offsets, n_offsets);
  if (st != SBDA_OK) return st;
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, L = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || L == 0) return SBDA_OK;
  if (!q.data || !k.data || !v.data || !grad_out.data || !lse || !grad_q.data || !grad_k.data ||
      !grad_v.data)
    return SBDA_ERR_INVALID;
  const int e = elem_size(dtype);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = tensors_vector_ok({&q, &k, &v, &grad_out, &grad_q, &grad_k, &grad_v}, B, L, D, e,
                                     {H, Hkv, Hkv, H, H, Hkv, Hkv});

  V2Plan p2;
  if (family == kFamilyAuto && plan_v2(offsets, n_offsets, L, D, e, H / Hkv, B, H, &p2)) {
    BwdV2Params p;
    memset(&p, 0, sizeof(p));
    p.G = 1;
    p.B = (int)B;
    p.H = (int)H;
    p.L = (int)L;
    p.D = (int)D;
    p.scale = scale;
    p.g = p2.g;
    p.q = arg_of(q);
    p.k = arg_of(k);
    p.v = arg_of(v);
    p.dout = arg_of(grad_out);
    p.dq = arg_of(grad_q);
    p.dk = arg_of(grad_k);
    p.dv = arg_of(grad_v);
    p.lse = lse;
    p.status = status_ptr();
    p.sh = single_shard(L, lse);
    BwdMaps maps;
    memset(&maps, 0, sizeof(maps));
    bool tma = vec;
    p.lse_box = p2.lse_box;
    p.lse_tx = p2.lse_box * 4;
    if (tma) {
      unsigned dummy;
      const int hz = p2.g.halo;
      const int lead = p2.g.mode == 2 ? p2.g.d : hz;  // K/V rows staged before a tile
      tma = encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, L, D, p2.pitch, p2.tile) &&
            encode_map(&maps.dT, &p.slots_d, grad_out, dtype, B, H, L, D, p2.pitch, p2.tile) &&
            encode_map(&maps.kT, &p.slots_k, k, dtype, B, H, L, D, p2.pitch, p2.tile) &&
            encode_map(&maps.vT, &p.slots_v, v, dtype, B, H, L, D, p2.pitch, p2.tile) &&
            encode_map(&maps.qH, &dummy, q, dtype, B, H, L, D, p2.pitch, hz) &&
            encode_map(&maps.dH, &dummy, grad_out, dtype, B, H, L, D, p2.pitch, hz) &&
            encode_map(&maps.kH, &dummy, k, dtype, B, H, L, D, p2.pitch, lead) &&
            encode_map(&maps.vH, &dummy, v, dtype, B, H, L, D, p2.pitch, lead);
      p.lse_tma = tma && encode_lse_map(&maps.lseT, lse, B * H, L, p2.lse_box);
    }
    return v2_backward(dtype, tma, maps, p, p2, s);
  }

  Plan pl;
  st = family == kFamilyUniform ? SBDA_ERR_UNSUPPORTED : make_plan(offsets, n_offsets, L, D, e, &pl);
  if (st == SBDA_ERR_UNSUPPORTED)  // several far offsets (or forced): the uniform kernels
    return uniform_backward(dtype, shape, offsets, n_offsets, scale, q, k, v, nullptr, grad_out, lse, grad_q,
                            grad_k, grad_v, vec, s);
  if (st != SBDA_OK) return st;
  BwdParams p;
  memset(&p, 0, sizeof(p));
  p.B = (int)B;
  p.H = (int)H;
  p.Hkv = (int)Hkv;
  p.G = (int)(H / Hkv);
  p.L = (int)L;
  p.D = (int)D;
  p.scale = scale;
  p.g = pl.g;
  p.q = arg_of(q);
  p.k = arg_of(k);
  p.v = arg_of(v);
  p.dout = arg_of(grad_out);
  p.dq = arg_of(grad_q);
  p.dk = arg_of(grad_k);
  p.dv = arg_of(grad_v);
  p.lse = lse;
  p.status = status_ptr();
  p.sh = single_shard(L, lse);
  BwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  bool tma = vec;
  if (tma) {
    unsigned dummy;
    tma = encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.dT, &p.slots_d, grad_out, dtype, B, H, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.kT, &p.slots_k, k, dtype, B, Hkv, L, D, pl.pitch, pl.tile) &&
          encode_map(&maps.vT, &p.slots_v, v, dtype, B, Hkv, L, D, pl.pitch, pl.tile);
    if (tma && pl.g.Hn > 0)
      tma = encode_map(&maps.qH, &dummy, q, dtype, B, H, L, D, pl.pitch, pl.g.Hn) &&
            encode_map(&maps.dH, &dummy, grad_out, dtype, B, H, L, D, pl.pitch, pl.g.Hn) &&
            encode_map(&maps.kH, &dummy, k, dtype, B, Hkv, L, D, pl.pitch, pl.g.Hn) &&
            encode_map(&maps.vH, &dummy, v, dtype, B, Hkv, L, D, pl.pitch, pl.g.Hn);
  }
  return v1_backward(dtype, tma, maps, p, pl, s);
}

extern "C" int sbda_b200_backward(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                  float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                                  sbda_tensor grad_out, const float* lse, sbda_tensor grad_q,
                                  sbda_tensor grad_k, sbda_tensor grad_v, void* stream) {
  return sbda_b200_backward_ex(kFamilyAuto, dtype, shape, offsets, n_offsets, scale, q, k, v, grad_out, lse,
                               grad_q, grad_k, grad_v, stream);
}

extern "C" int sbda_b200_forward_masked(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                        float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                                        const uint8_t* source_mask, sbda_tensor out, float* lse, void* stream) {
  int st = validate(dtype, shape, offsets, n_offsets);
  if (st != SBDA_OK) return st;
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, L = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || L == 0) return SBDA_OK;
  if (!q.data || !k.data || !v.data || !out.data || !lse || !source_mask) return SBDA_ERR_INVALID;
  const int e = elem_size(dtype);
  const bool vec = tensors_vector_ok({&q, &k, &v, &out}, B, L, D, e, {H, Hkv, Hkv, H});
  return uniform_forward(dtype, shape, offsets, n_offsets, scale, q, k, v, source_mask, out, lse, vec,
                         reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sbda_b200_backward_masked(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                         float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                                         const uint8_t* source_mask, sbda_tensor grad_out, const float* lse,
                                         sbda_tensor grad_q, sbda_tensor grad_k, sbda_tensor grad_v,
                                         void* stream) {
  int st = validate(dtype, shape, offsets, n_offsets);
  if (st != SBDA_OK) return st;
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, L = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || L == 0) return SBDA_OK;
  if (!q.data || !k.data || !v.data || !grad_out.data || !lse || !grad_q.data || !grad_k.data ||
      !grad_v.data || !source_mask)
    return SBDA_ERR_INVALID;
  const int e = elem_size(dtype);
  const bool vec = tensors_vector_ok({&q, &k, &v, &grad_out, &grad_q, &grad_k, &grad_v}, B, L, D, e,
                                     {H, Hkv, Hkv, H, H, Hkv, Hkv});
  return uniform_backward(dtype, shape, offsets, n_offsets, scale, q, k, v, source_mask, grad_out, lse, grad_q,
                          grad_k, grad_v, vec, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sbda_b200_device_status(uint32_t* flags_out, int reset) {
  unsigned value = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return SBDA_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&value, g_device_status, sizeof(value)) != cudaSuccess) return SBDA_ERR_CUDA;
  if (reset) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero)) != cudaSuccess) return SBDA_ERR_CUDA;
  }
  if (flags_out) *flags_out = value;
  return value ? SBDA_ERR_DEVICE : SBDA_OK;
}

// --------------------------------------------------------------------------
// Contiguous sequence shards
// --------------------------------------------------------------------------

namespace sbda {

// Plan of a sharded call: the general kernels' tiling, linear tile order, and
// every staged region inside one rank (shards and the far offset are tile
// multiples).  Returns a status.
int plan_sharded(const int32_t* offsets, int n, int64_t Ls, int64_t D, int e, int world, Plan* pl) {
  const int st = make_plan(offsets, n, Ls, D, e, pl);
  if (st != SBDA_OK) return st;
  if (world < 1 || world > kMaxShards) return SBDA_ERR_INVALID;
  if (Ls % pl->tile) return SBDA_ERR_UNSUPPORTED;
  if (pl->g.has_far && pl->g.f % pl->tile) return SBDA_ERR_UNSUPPORTED;
  if (pl->g.Hn > Ls) return SBDA_ERR_UNSUPPORTED;
  if ((int64_t)world * Ls > ((int64_t)1 << 31) - 1) return SBDA_ERR_UNSUPPORTED;
  pl->g.R = pl->g.A = pl->g.rem = 0;  // the far tile may live on another GPU: plain tile order
  return SBDA_OK;
}

ShardInfo shard_info(int rank, int world, int64_t Ls) {
  ShardInfo s;
  memset(&s, 0, sizeof(s));
  s.rank = rank;
  s.world = world;
  s.shard_len = (int)Ls;
  s.pos0 = (int)(rank * Ls);
  s.total_len = (int)(world * Ls);
  return s;
}

// Encodes one map per rank; all ranks' buffers must share one layout.
bool encode_ranks(CUtensorMap* maps, unsigned* slots, const sbda_tensor* ts, int world, int dtype, int64_t B,
                  int64_t H, int64_t L, int64_t D, int pitch, int rows) {
  unsigned first = 0;
  for (int r = 0; r < world; ++r) {
    unsigned s = 0;
    if (!vector_ok(ts[r], B, H, L, D, elem_size(dtype))) return false;
    if (!encode_map(&maps[r], &s, ts[r], dtype, B, H, L, D, pitch, rows)) return false;
    if (r == 0) first = s;
    else if (s != first) return false;
  }
  if (slots) *slots = first;
  return true;
}

}  // namespace sbda

extern "C" int sbda_b200_forward_sharded_ex(int family, int dtype, sbda_shape shape, const int32_t* offsets,
                                            int32_t n_offsets, float scale, int32_t rank, int32_t world,
                                            sbda_tensor q, const sbda_tensor* k_ranks, const sbda_tensor* v_ranks,
                                            sbda_tensor out, float* lse, void* stream) {
  if (!family_ok(family)) return SBDA_ERR_INVALID;
  int st = validate(dtype, shape, offsets, n_offsets);
  if (st != SBDA_OK) return st;
  if (world < 1 || world > kMaxShards || rank < 0 || rank >= world || !k_ranks || !v_ranks)
    return SBDA_ERR_INVALID;
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, Ls = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || Ls == 0) return SBDA_OK;
  if (!q.data || !out.data || !lse) return SBDA_ERR_INVALID;
  for (int r = 0; r < world; ++r)
    if (!k_ranks[r].data || !v_ranks[r].data) return SBDA_ERR_INVALID;
  // One shard is the whole sequence: the unsharded kernels (windowed where they apply).
  if (world == 1)
    return sbda_b200_forward_ex(family, dtype, shape, offsets, n_offsets, scale, q, k_ranks[0], v_ranks[0], out, lse,
                                stream);
  const int e = elem_size(dtype);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  {  // The windowed kernels, when they serve the schedule and every view suits the copy engine.
    V2Plan p2;
    if (family == kFamilyAuto && plan_v2(offsets, n_offsets, Ls, D, e, H / Hkv, B, H, &p2, world * Ls) &&
        Ls % p2.tile == 0 && vector_ok(q, B, H, Ls, D, e) && vector_ok(out, B, H, Ls, D, e)) {
      FwdV2Params p;
      memset(&p, 0, sizeof(p));
      p.G = 1;
      p.B = (int)B;
      p.H = (int)H;
      p.L = (int)Ls;
      p.D = (int)D;
      p.scale = scale;
      p.g = p2.g;
      p.q = arg_of(q);
      p.k = arg_of(k_ranks[rank]);
      p.v = arg_of(v_ranks[rank]);
      p.out = arg_of(out);
      p.lse = lse;
      p.status = status_ptr();
      p.sh = shard_info(rank, world, Ls);
      p.sh.lse[rank] = lse;
      ShardFwdMaps maps;
      memset(&maps, 0, sizeof(maps));
      if (encode_ranks(maps.kT, &p.slots_k, k_ranks, world, dtype, B, H, Ls, D, p2.pitch, p2.tile) &&
          encode_ranks(maps.vT, &p.slots_v, v_ranks, world, dtype, B, H, Ls, D, p2.pitch, p2.tile) &&
          encode_ranks(maps.kH, nullptr, k_ranks, world, dtype, B, H, Ls, D, p2.pitch, fwd_window_lead(p2.g, p2.tile)) &&
          encode_ranks(maps.vH, nullptr, v_ranks, world, dtype, B, H, Ls, D, p2.pitch, fwd_window_lead(p2.g, p2.tile)))
        return v2_forward_sharded(dtype, maps, p, p2, s);
    }
  }
  Plan pl;
  st = plan_sharded(offsets, n_offsets, Ls, D, e, world, &pl);
  if (st != SBDA_OK) return st;
  if (!vector_ok(q, B, H, Ls, D, e) || !vector_ok(out, B, H, Ls, D, e)) return SBDA_ERR_UNSUPPORTED;

  FwdParams p;
  memset(&p, 0, sizeof(p));
  p.B = (int)B;
  p.H = (int)H;
  p.Hkv = (int)Hkv;
  p.G = (int)(H / Hkv);
  p.L = (int)Ls;
  p.D = (int)D;
  p.scale = scale;
  p.g = pl.g;
  p.q = arg_of(q);
  p.k = arg_of(k_ranks[rank]);
  p.v = arg_of(v_ranks[rank]);
  p.out = arg_of(out);
  p.lse = lse;
  p.status = status_ptr();
  p.sh = shard_info(rank, world, Ls);
  p.sh.lse[rank] = lse;

  ShardFwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  bool ok = encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, Ls, D, pl.pitch, pl.tile) &&
            encode_ranks(maps.kT, &p.slots_k, k_ranks, world, dtype, B, Hkv, Ls, D, pl.pitch, pl.tile) &&
            encode_ranks(maps.vT, &p.slots_v, v_ranks, world, dtype, B, Hkv, Ls, D, pl.pitch, pl.tile);
  if (ok && pl.g.Hn > 0)
    ok = encode_ranks(maps.kH, nullptr, k_ranks, world, dtype, B, Hkv, Ls, D, pl.pitch, pl.g.Hn) &&
         encode_ranks(maps.vH, nullptr, v_ranks, world, dtype, B, Hkv, Ls, D, pl.pitch, pl.g.Hn);
  if (!ok) return SBDA_ERR_UNSUPPORTED;
  return v1_forward_sharded(dtype, maps, p, pl, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sbda_b200_backward_sharded_ex(int family, int dtype, sbda_shape shape, const int32_t* offsets,
                                             int32_t n_offsets, float scale, int32_t rank, int32_t world,
                                             const sbda_tensor* q_ranks, const sbda_tensor* k_ranks,
                                             const sbda_tensor* v_ranks, const sbda_tensor* grad_out_ranks,
                                             const float* const* lse_ranks, sbda_tensor grad_q, sbda_tensor grad_k,
                                             sbda_tensor grad_v, void* stream) {
  if (!family_ok(family)) return SBDA_ERR_INVALID;
  int st = validate(dtype, shape, offsets, n_offsets);
  if (st != SBDA_OK) return st;
  if (world < 1 || world > kMaxShards || rank < 0 || rank >= world || !q_ranks || !k_ranks || !v_ranks ||
      !grad_out_ranks || !lse_ranks)
    return SBDA_ERR_INVALID;
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, Ls = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || Ls == 0) return SBDA_OK;
  if (!grad_q.data || !grad_k.data || !grad_v.data) return SBDA_ERR_INVALID;
  for (int r = 0; r < world; ++r)
    if (!q_ranks[r].data || !k_ranks[r].data || !v_ranks[r].data || !grad_out_ranks[r].data || !lse_ranks[r])
      return SBDA_ERR_INVALID;
  if (world == 1)
    return sbda_b200_backward_ex(family, dtype, shape, offsets, n_offsets, scale, q_ranks[0], k_ranks[0],
                                 v_ranks[0], grad_out_ranks[0], lse_ranks[0], grad_q, grad_k, grad_v, stream);
  const int e = elem_size(dtype);
  {  // The windowed kernels, when they serve the schedule and every view suits the copy engine.
    V2Plan p2;
    if (family == kFamilyAuto && plan_v2(offsets, n_offsets, Ls, D, e, H / Hkv, B, H, &p2, world * Ls) &&
        Ls % p2.tile == 0 && vector_ok(grad_q, B, H, Ls, D, e) && vector_ok(grad_k, B, H, Ls, D, e) &&
        vector_ok(grad_v, B, H, Ls, D, e)) {
      BwdV2Params p;
      memset(&p, 0, sizeof(p));
      p.G = 1;
      p.B = (int)B;
      p.H = (int)H;
      p.L = (int)Ls;
      p.D = (int)D;
      p.scale = scale;
      p.g = p2.g;
      p.q = arg_of(q_ranks[rank]);
      p.k = arg_of(k_ranks[rank]);
      p.v = arg_of(v_ranks[rank]);
      p.dout = arg_of(grad_out_ranks[rank]);
      p.dq = arg_of(grad_q);
      p.dk = arg_of(grad_k);
      p.dv = arg_of(grad_v);
      p.lse = lse_ranks[rank];
      p.status = status_ptr();
      p.lse_box = p2.lse_box;
      p.sh = shard_info(rank, world, Ls);
      for (int r = 0; r < world; ++r) p.sh.lse[r] = lse_ranks[r];
      const int hz = p2.g.halo;
      const int lead = p2.g.mode == 2 ? p2.g.d : hz;
      ShardBwdMaps maps;
      memset(&maps, 0, sizeof(maps));
      // LSE rows by the copy engine: the tile's rows and the halo rows past it
      // (rounded up to 16 bytes), each box from its owner; else per-row loads.
      const int lse_halo = (hz + 3) / 4 * 4;
      p.lse_tma = 1;
      p.lse_tx = (p2.tile + lse_halo) * 4;
      for (int r = 0; r < world && p.lse_tma; ++r)
        p.lse_tma = encode_lse_map(&maps.lseT[r], lse_ranks[r], B * H, Ls, p2.tile) &&
                    encode_lse_map(&maps.lseH[r], lse_ranks[r], B * H, Ls, lse_halo);
      if (encode_ranks(maps.qT, &p.slots_q, q_ranks, world, dtype, B, H, Ls, D, p2.pitch, p2.tile) &&
          encode_ranks(maps.dT, &p.slots_d, grad_out_ranks, world, dtype, B, H, Ls, D, p2.pitch, p2.tile) &&
          encode_ranks(maps.kT, &p.slots_k, k_ranks, world, dtype, B, H, Ls, D, p2.pitch, p2.tile) &&
          encode_ranks(maps.vT, &p.slots_v, v_ranks, world, dtype, B, H, Ls, D, p2.pitch, p2.tile) &&
          encode_ranks(maps.qH, nullptr, q_ranks, world, dtype, B, H, Ls, D, p2.pitch, hz) &&
          encode_ranks(maps.dH, nullptr, grad_out_ranks, world, dtype, B, H, Ls, D, p2.pitch, hz) &&
          encode_ranks(maps.kH, nullptr, k_ranks, world, dtype, B, H, Ls, D, p2.pitch, lead) &&
          encode_ranks(maps.vH, nullptr, v_ranks, world, dtype, B, H, Ls, D, p2.pitch, lead))
        return v2_backward_sharded(dtype, maps, p, p2, reinterpret_cast<cudaStream_t>(stream));
    }
  }
  Plan pl;
  st = plan_sharded(offsets, n_offsets, Ls, D, e, world, &pl);
  if (st != SBDA_OK) return st;
  if (!vector_ok(grad_q, B, H, Ls, D, e) || !vector_ok(grad_k, B, Hkv, Ls, D, e) ||
      !vector_ok(grad_v, B, Hkv, Ls, D, e))
    return SBDA_ERR_UNSUPPORTED;

  BwdParams p;
  memset(&p, 0, sizeof(p));
  p.B = (int)B;
  p.H = (int)H;
  p.Hkv = (int)Hkv;
  p.G = (int)(H / Hkv);
  p.L = (int)Ls;
  p.D = (int)D;
  p.scale = scale;
  p.g = pl.g;
  p.q = arg_of(q_ranks[rank]);
  p.k = arg_of(k_ranks[rank]);
  p.v = arg_of(v_ranks[rank]);
  p.dout = arg_of(grad_out_ranks[rank]);
  p.dq = arg_of(grad_q);
  p.dk = arg_of(grad_k);
  p.dv = arg_of(grad_v);
  p.lse = lse_ranks[rank];
  p.status = status_ptr();
  p.sh = shard_info(rank, world, Ls);
  for (int r = 0; r < world; ++r) p.sh.lse[r] = lse_ranks[r];

  ShardBwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  bool ok = encode_ranks(maps.qT, &p.slots_q, q_ranks, world, dtype, B, H, Ls, D, pl.pitch, pl.tile) &&
            encode_ranks(maps.dT, &p.slots_d, grad_out_ranks, world, dtype, B, H, Ls, D, pl.pitch, pl.tile) &&
            encode_ranks(maps.kT, &p.slots_k, k_ranks, world, dtype, B, Hkv, Ls, D, pl.pitch, pl.tile) &&
            encode_ranks(maps.vT, &p.slots_v, v_ranks, world, dtype, B, Hkv, Ls, D, pl.pitch, pl.tile);
  if (ok && pl.g.Hn > 0)
    ok = encode_ranks(maps.qH, nullptr, q_ranks, world, dtype, B, H, Ls, D, pl.pitch, pl.g.Hn) &&
         encode_ranks(maps.dH, nullptr, grad_out_ranks, world, dtype, B, H, Ls, D, pl.pitch, pl.g.Hn) &&
         encode_ranks(maps.kH, nullptr, k_ranks, world, dtype, B, Hkv, Ls, D, pl.pitch, pl.g.Hn) &&
         encode_ranks(maps.vH, nullptr, v_ranks, world, dtype, B, Hkv, Ls, D, pl.pitch, pl.g.Hn);
  if (!ok) return SBDA_ERR_UNSUPPORTED;
  return v1_backward_sharded(dtype, maps, p, pl, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sbda_b200_forward_sharded(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                         float scale, int32_t rank, int32_t world, sbda_tensor q,
                                         const sbda_tensor* k_ranks, const sbda_tensor* v_ranks, sbda_tensor out,
                                         float* lse, void* stream) {
  return sbda_b200_forward_sharded_ex(kFamilyAuto, dtype, shape, offsets, n_offsets, scale, rank, world, q, k_ranks,
                                      v_ranks, out, lse, stream);
}

extern "C" int sbda_b200_backward_sharded(int dtype, sbda_shape shape, const int32_t* offsets,
                                          int32_t n_offsets, float scale, int32_t rank, int32_t world,
                                          const sbda_tensor* q_ranks, const sbda_tensor* k_ranks,
                                          const sbda_tensor* v_ranks, const sbda_tensor* grad_out_ranks,
                                          const float* const* lse_ranks, sbda_tensor grad_q, sbda_tensor grad_k,
                                          sbda_tensor grad_v, void* stream) {
  return sbda_b200_backward_sharded_ex(kFamilyAuto, dtype, shape, offsets, n_offsets, scale, rank, world, q_ranks,
                                       k_ranks, v_ranks, grad_out_ranks, lse_ranks, grad_q, grad_k, grad_v, stream);
}

// --------------------------------------------------------------------------
// Attention with the per-head RMSNorm + RoPE of q and k fused in
// --------------------------------------------------------------------------

namespace sbda {

// Shape-level eligibility of the fused entry points; fills the plan.
int normed_plan(int dtype, const sbda_shape& shape, const int32_t* offsets, int n, V2Plan* p2) {
  const int st = validate(dtype, shape, offsets, n);
  if (st != SBDA_OK) return st;
  if (shape.head_dim != 64 || shape.heads != shape.kv_heads) return SBDA_ERR_UNSUPPORTED;
  if (shape.batch == 0 || shape.heads == 0 || shape.length == 0) return SBDA_OK;
  if (!plan_v2(offsets, n, shape.length, shape.head_dim, elem_size(dtype), 1, shape.batch, shape.heads, p2))
    return SBDA_ERR_UNSUPPORTED;
  return v2_normed_plan_ok(*p2) ? SBDA_OK : SBDA_ERR_UNSUPPORTED;
}

// Norm weights (fp32 [64], 16-byte aligned) and tables ([rows, 32] in the
// element type, 16-byte aligned) of one tensor.
int normed_args(NormRopeArgs* a, const float* w, float eps, const void* cos_t, const void* sin_t,
                int64_t table_offset) {
  if (!w || !cos_t || !sin_t || table_offset < 0) return SBDA_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(cos_t) % 16 ||
      reinterpret_cast<uintptr_t>(sin_t) % 16)
    return SBDA_ERR_UNSUPPORTED;
  if (!(eps >= 0.f)) return SBDA_ERR_INVALID;
  a->w = w;
  a->cos_t = cos_t;
  a->sin_t = sin_t;
  a->table_offset = table_offset;
  a->eps = eps;
  return SBDA_OK;
}

}  // namespace sbda

extern "C" int sbda_b200_normed_supported(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets) {
  V2Plan p2;
  return normed_plan(dtype, shape, offsets, n_offsets, &p2) == SBDA_OK ? 1 : 0;
}

extern "C" int sbda_b200_forward_normed(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                        float scale, sbda_tensor q_raw, sbda_tensor k_raw, sbda_tensor v,
                                        const float* q_weight, float q_eps, const float* k_weight, float k_eps,
                                        const void* cos_table, const void* sin_table, int64_t table_offset,
                                        sbda_tensor out, float* lse, void* stream) {
  V2Plan p2;
  int st = normed_plan(dtype, shape, offsets, n_offsets, &p2);
  if (st != SBDA_OK) return st;
  const int64_t B = shape.batch, H = shape.heads, L = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || L == 0) return SBDA_OK;
  if (!q_raw.data || !k_raw.data || !v.data || !out.data || !lse) return SBDA_ERR_INVALID;
  FwdV2Params p;
  memset(&p, 0, sizeof(p));
  p.G = 1;
  if ((st = normed_args(&p.nq, q_weight, q_eps, cos_table, sin_table, table_offset)) != SBDA_OK) return st;
  if ((st = normed_args(&p.nk, k_weight, k_eps, cos_table, sin_table, table_offset)) != SBDA_OK) return st;
  const int e = elem_size(dtype);
  if (!tensors_vector_ok({&q_raw, &k_raw, &v, &out}, B, L, D, e, {H, H, H, H})) return SBDA_ERR_UNSUPPORTED;
  p.B = (int)B;
  p.H = (int)H;
  p.L = (int)L;
  p.D = (int)D;
  p.scale = scale;
  p.g = p2.g;
  p.q = arg_of(q_raw);
  p.k = arg_of(k_raw);
  p.v = arg_of(v);
  p.out = arg_of(out);
  p.lse = lse;
  p.status = status_ptr();
  p.sh = single_shard(L, lse);
  FwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  unsigned dummy;
  const int lead = fwd_window_lead(p2.g, p2.tile);
  if (!(encode_map(&maps.qT, &p.slots_q, q_raw, dtype, B, H, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.kT, &p.slots_k, k_raw, dtype, B, H, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.vT, &p.slots_v, v, dtype, B, H, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.kH, &dummy, k_raw, dtype, B, H, L, D, p2.pitch, lead) &&
        encode_map(&maps.vH, &dummy, v, dtype, B, H, L, D, p2.pitch, lead)))
    return SBDA_ERR_UNSUPPORTED;
  return v2_forward_normed(dtype, maps, p, p2, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int64_t sbda_b200_backward_normed_workspace_floats(int dtype, sbda_shape shape, const int32_t* offsets,
                                                              int32_t n_offsets) {
  V2Plan p2;
  if (normed_plan(dtype, shape, offsets, n_offsets, &p2) != SBDA_OK) return -1;
  if (shape.batch == 0 || shape.heads == 0 || shape.length == 0) return 0;
  return v2_normed_workspace_floats(p2.blocks_bwd);
}

extern "C" int sbda_b200_backward_normed(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                         float scale, sbda_tensor q_raw, sbda_tensor k_raw, sbda_tensor v,
                                         sbda_tensor grad_out, const float* lse, const float* q_weight, float q_eps,
                                         const float* k_weight, float k_eps, const void* cos_table,
                                         const void* sin_table, int64_t table_offset, sbda_tensor grad_q,
                                         sbda_tensor grad_k, sbda_tensor grad_v, float* grad_q_weight,
                                         float* grad_k_weight, float* workspace, int64_t workspace_floats,
                                         void* stream) {
  V2Plan p2;
  int st = normed_plan(dtype, shape, offsets, n_offsets, &p2);
  if (st != SBDA_OK) return st;
  const int64_t B = shape.batch, H = shape.heads, L = shape.length, D = shape.head_dim;
  if (!grad_q_weight || !grad_k_weight) return SBDA_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (B == 0 || H == 0 || L == 0) {  // empty: the weight gradients are zero
    if (cudaMemsetAsync(grad_q_weight, 0, 64 * sizeof(float), s) != cudaSuccess ||
        cudaMemsetAsync(grad_k_weight, 0, 64 * sizeof(float), s) != cudaSuccess)
      return SBDA_ERR_CUDA;
    return SBDA_OK;
  }
  if (!q_raw.data || !k_raw.data || !v.data || !grad_out.data || !lse || !grad_q.data || !grad_k.data ||
      !grad_v.data || !workspace)
    return SBDA_ERR_INVALID;
  if (workspace_floats < v2_normed_workspace_floats(p2.blocks_bwd)) return SBDA_ERR_INVALID;
  BwdV2Params p;
  memset(&p, 0, sizeof(p));
  p.G = 1;
  if ((st = normed_args(&p.nq, q_weight, q_eps, cos_table, sin_table, table_offset)) != SBDA_OK) return st;
  if ((st = normed_args(&p.nk, k_weight, k_eps, cos_table, sin_table, table_offset)) != SBDA_OK) return st;
  const int e = elem_size(dtype);
  if (!tensors_vector_ok({&q_raw, &k_raw, &v, &grad_out, &grad_q, &grad_k, &grad_v}, B, L, D, e,
                         {H, H, H, H, H, H, H}))
    return SBDA_ERR_UNSUPPORTED;
  p.B = (int)B;
  p.H = (int)H;
  p.L = (int)L;
  p.D = (int)D;
  p.scale = scale;
  p.g = p2.g;
  p.q = arg_of(q_raw);
  p.k = arg_of(k_raw);
  p.v = arg_of(v);
  p.dout = arg_of(grad_out);
  p.dq = arg_of(grad_q);
  p.dk = arg_of(grad_k);
  p.dv = arg_of(grad_v);
  p.lse = lse;
  p.status = status_ptr();
  p.sh = single_shard(L, lse);
  p.lse_box = p2.lse_box;
  p.lse_tx = p2.lse_box * 4;
  p.dw_partial = workspace;
  BwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  unsigned dummy;
  const int hz = p2.g.halo;
  const int lead = p2.g.mode == 2 ? p2.g.d : hz;
  if (!(encode_map(&maps.qT, &p.slots_q, q_raw, dtype, B, H, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.dT, &p.slots_d, grad_out, dtype, B, H, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.kT, &p.slots_k, k_raw, dtype, B, H, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.vT, &p.slots_v, v, dtype, B, H, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.qH, &dummy, q_raw, dtype, B, H, L, D, p2.pitch, hz) &&
        encode_map(&maps.dH, &dummy, grad_out, dtype, B, H, L, D, p2.pitch, hz) &&
        encode_map(&maps.kH, &dummy, k_raw, dtype, B, H, L, D, p2.pitch, lead) &&
        encode_map(&maps.vH, &dummy, v, dtype, B, H, L, D, p2.pitch, lead)))
    return SBDA_ERR_UNSUPPORTED;
  p.lse_tma = encode_lse_map(&maps.lseT, lse, B * H, L, p2.lse_box);
  return v2_backward_normed(dtype, maps, p, p2, grad_q_weight, grad_k_weight, workspace, s);
}

// --------------------------------------------------------------------------
// Grouped-query attention on the windowed backward
// --------------------------------------------------------------------------

extern "C" int64_t sbda_b200_backward_grouped_workspace_floats(sbda_shape shape) {
  if (shape.batch < 0 || shape.heads < 0 || shape.length < 0 || shape.head_dim < 1) return -1;
  return 2 * shape.batch * shape.heads * shape.length * shape.head_dim;
}

extern "C" int sbda_b200_backward_grouped(int dtype, sbda_shape shape, const int32_t* offsets, int32_t n_offsets,
                                          float scale, sbda_tensor q, sbda_tensor k, sbda_tensor v,
                                          sbda_tensor grad_out, const float* lse, sbda_tensor grad_q,
                                          sbda_tensor grad_k, sbda_tensor grad_v, float* workspace,
                                          int64_t workspace_floats, void* stream) {
  int st = validate(dtype, shape, offsets, n_offsets);
  if (st != SBDA_OK) return st;
  const int64_t B = shape.batch, H = shape.heads, Hkv = shape.kv_heads, L = shape.length, D = shape.head_dim;
  if (B == 0 || H == 0 || L == 0) return SBDA_OK;
  if (!q.data || !k.data || !v.data || !grad_out.data || !lse || !grad_q.data || !grad_k.data || !grad_v.data)
    return SBDA_ERR_INVALID;
  auto general = [&] {
    return sbda_b200_backward_ex(kFamilyAuto, dtype, shape, offsets, n_offsets, scale, q, k, v, grad_out, lse,
                                 grad_q, grad_k, grad_v, stream);
  };
  if (H == Hkv) return general();  // MHA: the windowed backward writes dK/dV itself
  if (!workspace || workspace_floats < sbda_b200_backward_grouped_workspace_floats(shape) ||
      reinterpret_cast<uintptr_t>(workspace) % 16)
    return SBDA_ERR_INVALID;
  const int e = elem_size(dtype);
  V2Plan p2;
  const bool vec = tensors_vector_ok({&q, &k, &v, &grad_out, &grad_q}, B, L, D, e, {H, Hkv, Hkv, H, H});
  // The walk is planned per query head as for MHA; K/V rows come from kv head h / G.
  if (!vec || D % 8 || !plan_v2(offsets, n_offsets, L, D, e, 1, B, H, &p2) || !v2_grouped_plan_ok(p2))
    return general();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  BwdV2Params p;
  memset(&p, 0, sizeof(p));
  p.G = (int)(H / Hkv);
  p.B = (int)B;
  p.H = (int)H;
  p.L = (int)L;
  p.D = (int)D;
  p.scale = scale;
  p.g = p2.g;
  p.q = arg_of(q);
  p.k = arg_of(k);
  p.v = arg_of(v);
  p.dout = arg_of(grad_out);
  p.dq = arg_of(grad_q);
  // fp32 per-query-head partials: [2][B, H, L, D], contiguous.
  const int64_t part = B * H * L * D;
  p.dk = TensorArg{workspace, H * L * D, L * D, D, 1};
  p.dv = TensorArg{workspace + part, H * L * D, L * D, D, 1};
  p.lse = lse;
  p.status = status_ptr();
  p.sh = single_shard(L, lse);
  p.lse_box = p2.lse_box;
  p.lse_tx = p2.lse_box * 4;
  BwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  unsigned dummy;
  const int hz = p2.g.halo;
  const int lead = p2.g.mode == 2 ? p2.g.d : hz;
  if (!(encode_map(&maps.qT, &p.slots_q, q, dtype, B, H, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.dT, &p.slots_d, grad_out, dtype, B, H, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.kT, &p.slots_k, k, dtype, B, Hkv, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.vT, &p.slots_v, v, dtype, B, Hkv, L, D, p2.pitch, p2.tile) &&
        encode_map(&maps.qH, &dummy, q, dtype, B, H, L, D, p2.pitch, hz) &&
        encode_map(&maps.dH, &dummy, grad_out, dtype, B, H, L, D, p2.pitch, hz) &&
        encode_map(&maps.kH, &dummy, k, dtype, B, Hkv, L, D, p2.pitch, lead) &&
        encode_map(&maps.vH, &dummy, v, dtype, B, Hkv, L, D, p2.pitch, lead)))
    return general();
  p.lse_tma = encode_lse_map(&maps.lseT, lse, B * H, L, p2.lse_box);
  st = v2_backward_grouped(dtype, maps, p, p2, workspace, (int)Hkv, arg_of(grad_k), arg_of(grad_v), s);
  return st == SBDA_ERR_UNSUPPORTED ? general() : st;
}
