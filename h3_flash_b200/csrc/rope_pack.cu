// Per-head QK RMSNorm + partial rotate-half RoPE, fused with the packed-Ulysses
// destination-major QKV pack; plus the standalone pack and head-merge relayouts.
//
// Head rows of D=128 bf16 are handled by D/8 lanes (16 lanes, two head rows per
// warp), 16 bytes per lane. The rotate-half partner of column c (c < rot) is
// c +/- rot/2; when rot/2 is a multiple of 8 the partner chunk sits rot/16 lanes
// away in the same head row and is fetched with a shuffle, otherwise it is read
// back from a per-warp shared-memory copy of the normalised row.
//
// Semantics: src/h3_flash/runtime/kernels/fusions.py:125-175 (norm + RoPE),
// src/h3_flash/runtime/parallel/relayout.py:10-67 (pack / merge).
#include <cstdio>

#include "common.cuh"

namespace h3b {
namespace {

// Normalise + rope one 8-column chunk owned by this lane. `v` holds the chunk's
// raw values on entry and the output on exit. All lanes of the warp must call
// this together (shuffles); `active` marks lanes that own a real chunk.
template <int D, bool kShufflePartner>
__device__ __forceinline__ void norm_rope_chunk(float (&v)[8], const __nv_bfloat16* weight,
                                                const float* cos_row, const float* sin_row,
                                                int rot, float eps, int sublane,
                                                float* smem_row) {
  constexpr int L = D / 8;  // lanes per head row
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
  // Reduce across the L lanes of this head row.
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)D + eps);
  const int col = sublane * 8;
  f8 w = unpack8(ld_cached(weight + col));
  float n[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) n[j] = v[j] * r * w.v[j];
  if (rot == 0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = n[j];
    return;
  }
  const int half = rot >> 1;
  float p[8];
  if (kShufflePartner) {
    const int dl = half >> 3;
    const int lane = threadIdx.x & 31;
    const int src = (col < half) ? lane + dl : lane - dl;
    const int src_ok = (col < rot) ? src : lane;
#pragma unroll
    for (int j = 0; j < 8; ++j) p[j] = __shfl_sync(0xffffffffu, n[j], src_ok);
    if (col < rot) {
      const float sgn = (col < half) ? -1.f : 1.f;
      const float4 c0 = __ldg(reinterpret_cast<const float4*>(cos_row + col));
      const float4 c1 = __ldg(reinterpret_cast<const float4*>(cos_row + col + 4));
      const float4 s0 = __ldg(reinterpret_cast<const float4*>(sin_row + col));
      const float4 s1 = __ldg(reinterpret_cast<const float4*>(sin_row + col + 4));
      const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = n[j] * cs[j] + (sgn * p[j]) * sn[j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = n[j];
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) smem_row[col + j] = n[j];
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = col + j;
      if (c < rot) {
        const bool first = c < half;
        const float pv = smem_row[first ? c + half : c - half];
        const float rotated = first ? -pv : pv;
        v[j] = n[j] * __ldg(cos_row + c) + rotated * __ldg(sin_row + c);
      } else {
        v[j] = n[j];
      }
    }
    __syncwarp();
  }
}

// Both kernels below flatten their work into head rows; a group of L = D/8
// lanes owns one head row per item and every thread keeps kItems items in
// flight (all loads issued before the first reduction) so enough bytes are
// outstanding per SM to cover HBM latency.
constexpr int kItems = 4;

// ---- standalone fused_qknorm_rope: x, out contiguous [B*S*H, D] -------------

template <int D, bool kShuffle>
__global__ void __launch_bounds__(256) qknorm_rope_kernel(__nv_bfloat16* out,
                                                         const __nv_bfloat16* x,
                                                         const __nv_bfloat16* weight,
                                                         const float* cos, const float* sin,
                                                         int64_t nrows, int64_t heads,
                                                         int64_t seq, int rot, float eps) {
  constexpr int L = D / 8;
  constexpr int G = 256 / L;  // head rows per CTA pass
  __shared__ float smem[kShuffle ? 1 : G * D];
  const int sub = threadIdx.x % L;
  const int slot = threadIdx.x / L;
  const int64_t base = (int64_t)blockIdx.x * G * kItems;
  uint4 raw[kItems];
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int64_t hr = base + k * G + slot;
    const int64_t hr_c = hr < nrows ? hr : nrows - 1;  // inactive lanes still join the shuffles
    raw[k] = ld_stream(x + hr_c * D + sub * 8);
  }
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int64_t hr = base + k * G + slot;
    const int64_t hr_c = hr < nrows ? hr : nrows - 1;
    const int64_t token = (hr_c / heads) % seq;
    f8 in = unpack8(raw[k]);
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = in.v[j];
    norm_rope_chunk<D, kShuffle>(v, weight, cos + token * rot, sin + token * rot, rot, eps, sub,
                                 kShuffle ? nullptr : smem + slot * D);
    if (hr < nrows) st_stream(out + hr * D + sub * 8, pack8(v));
  }
}

// ---- fused q/k norm + rope + destination-major pack -------------------------
//
// Work items are the rows * 3H head rows (row-major: q heads, k heads, v heads
// of token 0, then token 1, ...). Each group of L lanes takes kItems items
// spaced G apart.
template <int D, bool kShuffle>
__global__ void __launch_bounds__(256) qknorm_rope_pack_kernel(
    __nv_bfloat16* send, const __nv_bfloat16* q, const __nv_bfloat16* k,
    const __nv_bfloat16* v, int64_t q_stride, int64_t k_stride, int64_t v_stride,
    const __nv_bfloat16* wq, const __nv_bfloat16* wk, const float* cos, const float* sin,
    int64_t rows, int heads, int hl, int rot, float q_eps, float k_eps) {
  constexpr int L = D / 8;
  constexpr int G = 256 / L;
  __shared__ float smem[kShuffle ? 1 : G * D];
  const int sub = threadIdx.x % L;
  const int slot = threadIdx.x / L;
  const int per_row = 3 * heads;
  const int64_t total = rows * per_row;
  const int64_t base = (int64_t)blockIdx.x * G * kItems;
  uint4 raw[kItems];
  int row_of[kItems], item_of[kItems];
#pragma unroll
  for (int it = 0; it < kItems; ++it) {
    int64_t w = base + it * G + slot;
    if (w >= total) w = total - 1;  // inactive lanes still join the shuffles
    const int w32 = (int)w;  // total < 2^31 (checked by the launcher)
    const int row = w32 / per_row;
    const int item = w32 - row * per_row;
    row_of[it] = row;
    item_of[it] = item;
    const int part = item / heads;
    const int g = item - part * heads;
    const __nv_bfloat16* src = part == 0   ? q + row * q_stride
                               : part == 1 ? k + row * k_stride
                                           : v + row * v_stride;
    raw[it] = ld_stream(src + (int64_t)g * D + sub * 8);
  }
#pragma unroll
  for (int it = 0; it < kItems; ++it) {
    const int64_t w = base + it * G + slot;
    const int row = row_of[it];
    const int part = item_of[it] / heads;  // 0 = q, 1 = k, 2 = v
    const int g = item_of[it] - part * heads;
    f8 in = unpack8(raw[it]);
    // Head rows of different parts share a warp: the warp-collective norm runs
    // for every lane and v rows store their raw bits unchanged.
    float nv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) nv[j] = in.v[j];
    norm_rope_chunk<D, kShuffle>(nv, part == 1 ? wk : wq, cos + (int64_t)row * rot,
                                 sin + (int64_t)row * rot, rot, part == 1 ? k_eps : q_eps, sub,
                                 kShuffle ? nullptr : smem + slot * D);
    if (w < total) {
      const int dst = g / hl;
      const int lh = g - dst * hl;
      __nv_bfloat16* o =
          send + (((int64_t)dst * rows + row) * hl + lh) * (3 * D) + part * D + sub * 8;
      st_stream(o, part == 2 ? raw[it] : pack8(nv));
    }
  }
}

// ---- fast path: one warp per token, partner chunks owned by the same lane ------
//
// For head_dim D and rotary_dim rot with rot % 16 == 0 and (D - rot) % 16 == 0,
// a head row is split into D/16 lane-owned chunk pairs of 8 columns: lane
// l < rot/16 owns chunk l and its rotate-half partner chunk l + rot/16; the
// remaining lanes own two consecutive pass-through chunks above rot. So the
// rotation needs no cross-lane data, and the norm's sum of squares is a
// (D/16)-lane shuffle reduction. One warp walks all heads of one token, so the
// QK-norm weights and the token's cos/sin stay in registers across heads; v
// head rows are a plain 16-byte copy.
template <int D>
struct PairLanes {
  static constexpr int L = D / 16;  // lanes per head row
  static constexpr int R = 32 / L;  // head rows per warp pass
};

template <int D>
__device__ __forceinline__ void lane_chunks(int sub, int rot, int& c0, int& c1, bool& pair) {
  const int np = rot / 16;
  if (sub < np) {
    c0 = sub;
    c1 = sub + np;
    pair = true;
  } else {
    c0 = rot / 8 + 2 * (sub - np);
    c1 = c0 + 1;
    pair = false;
  }
}

// Normalise (fp32 sum over the head row) + rotate one head row's two chunks.
template <int D>
__device__ __forceinline__ void norm_rope_pair(const uint4& ra, const uint4& rb, const f8& w0,
                                               const f8& w1, const float (&cs0)[8],
                                               const float (&sn0)[8], const float (&cs1)[8],
                                               const float (&sn1)[8], bool pair, float eps,
                                               uint4& oa, uint4& ob) {
  constexpr int L = PairLanes<D>::L;
  f8 a = unpack8(ra), b = unpack8(rb);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += a.v[j] * a.v[j] + b.v[j] * b.v[j];
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)D + eps);
  float na[8], nb[8], xa[8], xb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    na[j] = a.v[j] * r * w0.v[j];
    nb[j] = b.v[j] * r * w1.v[j];
  }
  if (pair) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      xa[j] = na[j] * cs0[j] + (-nb[j]) * sn0[j];  // first half takes -partner
      xb[j] = nb[j] * cs1[j] + na[j] * sn1[j];
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      xa[j] = na[j];
      xb[j] = nb[j];
    }
  }
  oa = pack8(xa);
  ob = pack8(xb);
}

template <int D>
__device__ __forceinline__ void load_rope_row(const float* cos_row, const float* sin_row, int c0,
                                              int c1, bool pair, float (&cs0)[8], float (&sn0)[8],
                                              float (&cs1)[8], float (&sn1)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) cs0[j] = sn0[j] = cs1[j] = sn1[j] = 0.f;
  if (!pair) return;
  const float4* c0p = reinterpret_cast<const float4*>(cos_row + 8 * c0);
  const float4* s0p = reinterpret_cast<const float4*>(sin_row + 8 * c0);
  const float4* c1p = reinterpret_cast<const float4*>(cos_row + 8 * c1);
  const float4* s1p = reinterpret_cast<const float4*>(sin_row + 8 * c1);
  float4 t;
#define H3B_F8(dst, src)          \
  t = __ldg(src);                 \
  dst[0] = t.x, dst[1] = t.y, dst[2] = t.z, dst[3] = t.w; \
  t = __ldg(src + 1);             \
  dst[4] = t.x, dst[5] = t.y, dst[6] = t.z, dst[7] = t.w;
  H3B_F8(cs0, c0p) H3B_F8(sn0, s0p) H3B_F8(cs1, c1p) H3B_F8(sn1, s1p)
#undef H3B_F8
}

constexpr int kTokWarps = 8;  // tokens (warps) per CTA

// Where the packed head rows go. LocalSend is the destination-major send buffer
// [W, rows, hl, 3D] that an all-to-all then exchanges; PeerRecv is every rank's
// receive buffer [S_total, hl, 3D] (this rank's own included), mapped into this
// process over NVLink, so the store itself is the exchange: row `row` of this
// rank lands at global row row_offset + row of the owner of its head.
struct LocalSend {
  __nv_bfloat16* send;
  int64_t rows;
  int hl;
  template <int D>
  __device__ __forceinline__ __nv_bfloat16* at(int64_t row, int g, int part) const {
    const int dst = g / hl, lh = g - dst * hl;
    return send + (((int64_t)dst * rows + row) * hl + lh) * (3 * D) + part * D;
  }
  __device__ __forceinline__ void store(void* p, uint4 v) const { st_stream(p, v); }
  __device__ __forceinline__ void finish() const {}
};

struct PeerRecv {
  PeerPtrs recv;
  int64_t row_offset;
  int hl;
  template <int D>
  __device__ __forceinline__ __nv_bfloat16* at(int64_t row, int g, int part) const {
    const int dst = g / hl, lh = g - dst * hl;
    return reinterpret_cast<__nv_bfloat16*>(peer_at(recv, dst)) +
           ((row_offset + row) * hl + lh) * (3 * D) + part * D;
  }
  __device__ __forceinline__ void store(void* p, uint4 v) const {
    *reinterpret_cast<uint4*>(p) = v;
  }
  // Peers read these rows after a cross-rank barrier; order the stores first.
  __device__ __forceinline__ void finish() const { __threadfence_system(); }
};

template <int D, class Dst>
__global__ void __launch_bounds__(kTokWarps * 32) qknorm_rope_pack_tok(
    Dst out, const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, int64_t q_stride, int64_t k_stride, int64_t v_stride,
    const __nv_bfloat16* __restrict__ wq, const __nv_bfloat16* __restrict__ wk,
    const float* __restrict__ cos, const float* __restrict__ sin, int64_t rows, int heads,
    int rot, float q_eps, float k_eps) {
  constexpr int L = PairLanes<D>::L;
  constexpr int R = PairLanes<D>::R;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kTokWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int sub = lane % L, slot = lane / L;
  int c0, c1;
  bool pair;
  lane_chunks<D>(sub, rot, c0, c1, pair);
  const f8 wq0 = unpack8(ld_cached(wq + 8 * c0)), wq1 = unpack8(ld_cached(wq + 8 * c1));
  const f8 wk0 = unpack8(ld_cached(wk + 8 * c0)), wk1 = unpack8(ld_cached(wk + 8 * c1));
  float cs0[8], sn0[8], cs1[8], sn1[8];
  load_rope_row<D>(cos + row * rot, sin + row * rot, c0, c1, pair, cs0, sn0, cs1, sn1);
  const __nv_bfloat16* qr = q + row * q_stride;
  const __nv_bfloat16* kr = k + row * k_stride;
  const __nv_bfloat16* vr = v + row * v_stride;
  auto dst_row = [&](int g, int part) { return out.template at<D>(row, g, part); };
  // q and k head rows: 2H of them, R per pass, 2 passes in flight.
  const int n_qk = 2 * heads;
  for (int it = 0; it < n_qk; it += 2 * R) {
    uint4 ra[2], rb[2];
    int hr[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      hr[u] = it + u * R + slot;
      const int h = hr[u] < n_qk ? hr[u] : n_qk - 1;  // idle lanes still join the shuffles
      const __nv_bfloat16* src = (h < heads ? qr + h * D : kr + (h - heads) * D);
      ra[u] = ld_stream(src + 8 * c0);
      rb[u] = ld_stream(src + 8 * c1);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const bool is_k = (hr[u] < n_qk ? hr[u] : n_qk - 1) >= heads;
      uint4 oa, ob;
      norm_rope_pair<D>(ra[u], rb[u], is_k ? wk0 : wq0, is_k ? wk1 : wq1, cs0, sn0, cs1, sn1, pair,
                        is_k ? k_eps : q_eps, oa, ob);
      if (hr[u] < n_qk) {
        const int g = is_k ? hr[u] - heads : hr[u];
        __nv_bfloat16* o = dst_row(g, is_k ? 1 : 0);
        out.store(o + 8 * c0, oa);
        out.store(o + 8 * c1, ob);
      }
    }
  }
  // v head rows: copy, 16 bytes per lane, 4 copies in flight.
  constexpr int C = D / 8;  // chunks per head row
  const int n_v = heads * C;
  for (int base = 0; base < n_v; base += 4 * 32) {
    uint4 val[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int cidx = base + u * 32 + lane;
      if (cidx < n_v) val[u] = ld_stream(vr + (int64_t)cidx * 8);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int cidx = base + u * 32 + lane;
      if (cidx < n_v) {
        const int g = cidx / C, cc = cidx - g * C;
        out.store(dst_row(g, 2) + 8 * cc, val[u]);
      }
    }
  }
  out.finish();
}

// Standalone fused_qknorm_rope on contiguous [B*S*H, D]: one warp per token
// (B*S tokens, H heads each), cos/sin row = token % S.
template <int D>
__global__ void __launch_bounds__(kTokWarps * 32) qknorm_rope_tok(
    __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ weight, const float* __restrict__ cos,
    const float* __restrict__ sin, int64_t tokens, int heads, int64_t seq, int rot, float eps) {
  constexpr int L = PairLanes<D>::L;
  constexpr int R = PairLanes<D>::R;
  const int lane = threadIdx.x & 31;
  const int64_t tok = (int64_t)blockIdx.x * kTokWarps + (threadIdx.x >> 5);
  if (tok >= tokens) return;
  const int sub = lane % L, slot = lane / L;
  int c0, c1;
  bool pair;
  lane_chunks<D>(sub, rot, c0, c1, pair);
  const f8 w0 = unpack8(ld_cached(weight + 8 * c0)), w1 = unpack8(ld_cached(weight + 8 * c1));
  float cs0[8], sn0[8], cs1[8], sn1[8];
  const int64_t s_idx = tok % seq;
  load_rope_row<D>(cos + s_idx * rot, sin + s_idx * rot, c0, c1, pair, cs0, sn0, cs1, sn1);
  const __nv_bfloat16* xr = x + tok * heads * D;
  __nv_bfloat16* orow = out + tok * heads * D;
  for (int it = 0; it < heads; it += 2 * R) {
    uint4 ra[2], rb[2];
    int hr[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      hr[u] = it + u * R + slot;
      const int h = hr[u] < heads ? hr[u] : heads - 1;
      ra[u] = ld_stream(xr + h * D + 8 * c0);
      rb[u] = ld_stream(xr + h * D + 8 * c1);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      uint4 oa, ob;
      norm_rope_pair<D>(ra[u], rb[u], w0, w1, cs0, sn0, cs1, sn1, pair, eps, oa, ob);
      if (hr[u] < heads) {
        st_stream(orow + hr[u] * D + 8 * c0, oa);
        st_stream(orow + hr[u] * D + 8 * c1, ob);
      }
    }
  }
}

// ---- pack_qkv_destination_major (no arithmetic) ----------------------------

template <int D>
__global__ void __launch_bounds__(256) pack_qkv_kernel(
    __nv_bfloat16* out, const __nv_bfloat16* q, const __nv_bfloat16* k,
    const __nv_bfloat16* v, int64_t rows, int heads, int hl, int64_t qr, int64_t qh,
    int64_t kr, int64_t kh, int64_t vr, int64_t vh) {
  constexpr int C = D / 8;  // chunks per head row
  const int64_t row = blockIdx.x;
  const int per_row = heads * 3 * C;
  for (int j = threadIdx.x; j < per_row; j += 256) {
    const int c = j % C;
    const int t = j / C;
    const int part = t % 3;
    const int g = t / 3;
    const __nv_bfloat16* src = part == 0   ? q + row * qr + g * qh
                               : part == 1 ? k + row * kr + g * kh
                                           : v + row * vr + g * vh;
    const int dst = g / hl, lh = g - dst * hl;
    __nv_bfloat16* o = out + (((int64_t)dst * rows + row) * hl + lh) * (3 * D) + part * D;
    st_stream(o + c * 8, ld_stream(src + c * 8));
  }
}

// Generic scalar pack for strides / widths the vector kernel cannot address.
__global__ void pack_qkv_scalar(__nv_bfloat16* out, const __nv_bfloat16* q,
                                const __nv_bfloat16* k, const __nv_bfloat16* v, int64_t rows,
                                int64_t heads, int64_t hl, int64_t D, int64_t qr, int64_t qh,
                                int64_t kr, int64_t kh, int64_t vr, int64_t vh) {
  const int64_t total = rows * heads * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = i % D;
    const int64_t slot = i / D;
    const int64_t lh = slot % hl;
    const int64_t rs = slot / hl;
    const int64_t row = rs % rows;
    const int64_t dst = rs / rows;
    const int64_t g = dst * hl + lh;
    const int64_t base = slot * 3 * D + d;
    out[base] = q[row * qr + g * qh + d];
    out[base + D] = k[row * kr + g * kh + d];
    out[base + 2 * D] = v[row * vr + g * vh + d];
  }
}

// ---- merge_heads: out[row, src, :] = x[src, row, :] ------------------------

__global__ void __launch_bounds__(256) merge_heads_vec(__nv_bfloat16* out,
                                                      const __nv_bfloat16* x, int64_t world,
                                                      int64_t rows, int64_t inner8) {
  // One CTA per output row: copies world * inner contiguous output values.
  const int64_t row = blockIdx.x;
  const int64_t per_row = world * inner8;
  for (int64_t j = threadIdx.x; j < per_row; j += 256) {
    const int64_t src = j / inner8;
    const int64_t c = j - src * inner8;
    st_stream(out + (row * per_row + j) * 8, ld_stream(x + ((src * rows + row) * inner8 + c) * 8));
  }
}

__global__ void merge_heads_scalar(__nv_bfloat16* out, const __nv_bfloat16* x, int64_t world,
                                   int64_t rows, int64_t inner) {
  const int64_t total = world * rows * inner;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tail = i % inner;
    const int64_t slot = i / inner;
    const int64_t src = slot % world;
    const int64_t row = slot / world;
    out[i] = x[(src * rows + row) * inner + tail];
  }
}

template <int D, bool kShuffle>
void launch_qkrope(__nv_bfloat16* out, const __nv_bfloat16* x, const __nv_bfloat16* w,
                   const float* cos, const float* sin, int64_t nrows, int64_t heads,
                   int64_t seq, int rot, float eps, cudaStream_t s) {
  constexpr int kRowsPerCta = 256 / (D / 8) * kItems;
  const int64_t grid = (nrows + kRowsPerCta - 1) / kRowsPerCta;
  qknorm_rope_kernel<D, kShuffle><<<(unsigned)grid, 256, 0, s>>>(out, x, w, cos, sin, nrows,
                                                                 heads, seq, rot, eps);
}

}  // namespace
}  // namespace h3b

using h3b::aligned16;

extern "C" int h3b_qknorm_rope(void* out, const void* x, const void* weight, const float* cos,
                               const float* sin, int64_t batch, int64_t seq, int64_t heads,
                               int64_t head_dim, int64_t rotary_dim, float eps,
                               h3b_stream_t stream) {
  H3B_REQUIRE(batch >= 0 && seq >= 0 && heads >= 0, "qknorm_rope: negative shape");
  H3B_REQUIRE(rotary_dim >= 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0,
              "fused qknorm+rope requires an even rotary dimension no wider than the head, "
              "got rotary_dim=%lld, head_dim=%lld",
              (long long)rotary_dim, (long long)head_dim);
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) {
    h3b::set_error("qknorm_rope: head_dim must be 64, 128 or 256");
    return H3B_ERR_UNSUPPORTED;
  }
  const int64_t nrows = batch * seq * heads;
  if (nrows == 0) return H3B_OK;
  H3B_REQUIRE(aligned16(x) && aligned16(out) && aligned16(weight),
              "qknorm_rope: x, out and weight must be 16-byte aligned");
  const bool shuffle = rotary_dim % 16 == 0 && aligned16(cos) && aligned16(sin);
  const int rot = (int)rotary_dim;
  auto* o = (__nv_bfloat16*)out;
  auto* xi = (const __nv_bfloat16*)x;
  auto* w = (const __nv_bfloat16*)weight;
  if (shuffle && (head_dim - rotary_dim) % 16 == 0 && heads <= 0x7fffffff) {
    const int64_t tokens = batch * seq;
    const unsigned grid = (unsigned)((tokens + h3b::kTokWarps - 1) / h3b::kTokWarps);
#define H3B_QT(DD)                                                                          \
  if (head_dim == DD)                                                                       \
    h3b::qknorm_rope_tok<DD><<<grid, h3b::kTokWarps * 32, 0, stream>>>(o, xi, w, cos, sin,    \
                                                                      tokens, (int)heads,   \
                                                                      seq, rot, eps);
    H3B_QT(64) H3B_QT(128) H3B_QT(256)
#undef H3B_QT
    return h3b::check_launch("h3b_qknorm_rope");
  }
#define H3B_QK(DD)                                                                         \
  if (head_dim == DD) {                                                                    \
    if (shuffle)                                                                           \
      h3b::launch_qkrope<DD, true>(o, xi, w, cos, sin, nrows, heads, seq, rot, eps, stream); \
    else                                                                                   \
      h3b::launch_qkrope<DD, false>(o, xi, w, cos, sin, nrows, heads, seq, rot, eps, stream); \
  }
  H3B_QK(64) H3B_QK(128) H3B_QK(256)
#undef H3B_QK
  return h3b::check_launch("h3b_qknorm_rope");
}

extern "C" int h3b_qknorm_rope_pack(void* send, const void* q, const void* k, const void* v,
                                    int64_t q_row_stride, int64_t k_row_stride,
                                    int64_t v_row_stride, const void* q_weight,
                                    const void* k_weight, const float* cos, const float* sin,
                                    int64_t rows, int64_t heads, int64_t head_dim,
                                    int64_t rotary_dim, int64_t world, float q_eps,
                                    float k_eps, h3b_stream_t stream) {
  H3B_REQUIRE(rows >= 0 && heads > 0 && world > 0, "qknorm_rope_pack: bad shape");
  H3B_REQUIRE(heads % world == 0, "heads (%lld) must divide Ulysses degree (%lld)",
              (long long)heads, (long long)world);
  H3B_REQUIRE(rotary_dim >= 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0,
              "fused qknorm+rope requires an even rotary dimension no wider than the head, "
              "got rotary_dim=%lld, head_dim=%lld",
              (long long)rotary_dim, (long long)head_dim);
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) {
    h3b::set_error("qknorm_rope_pack: head_dim must be 64, 128 or 256");
    return H3B_ERR_UNSUPPORTED;
  }
  if (rows == 0) return H3B_OK;
  H3B_REQUIRE(rows * 3 * heads <= 0x7fffffffLL, "qknorm_rope_pack: too many rows");
  H3B_REQUIRE(aligned16(send) && aligned16(q) && aligned16(k) && aligned16(v) &&
                  aligned16(q_weight) && aligned16(k_weight) && q_row_stride % 8 == 0 &&
                  k_row_stride % 8 == 0 && v_row_stride % 8 == 0,
              "qknorm_rope_pack: tensors must be 16-byte aligned with row strides "
              "divisible by 8");
  const bool shuffle = rotary_dim % 16 == 0 && aligned16(cos) && aligned16(sin);
  const int hl = (int)(heads / world);
  auto* o = (__nv_bfloat16*)send;
  if (shuffle && (head_dim - rotary_dim) % 16 == 0) {
    const unsigned grid = (unsigned)((rows + h3b::kTokWarps - 1) / h3b::kTokWarps);
#define H3B_QPT(DD)                                                                         \
  if (head_dim == DD)                                                                       \
    h3b::qknorm_rope_pack_tok<DD><<<grid, h3b::kTokWarps * 32, 0, stream>>>(                  \
        h3b::LocalSend{o, rows, hl}, (const __nv_bfloat16*)q, (const __nv_bfloat16*)k,    \
        (const __nv_bfloat16*)v, q_row_stride, k_row_stride, v_row_stride,                 \
        (const __nv_bfloat16*)q_weight, (const __nv_bfloat16*)k_weight, cos, sin, rows,    \
        (int)heads, (int)rotary_dim, q_eps, k_eps);
    H3B_QPT(64) H3B_QPT(128) H3B_QPT(256)
#undef H3B_QPT
    return h3b::check_launch("h3b_qknorm_rope_pack");
  }
  const int64_t total_items = rows * 3 * heads;
#define H3B_QKP(DD, SH)                                                                   \
  h3b::qknorm_rope_pack_kernel<DD, SH><<<(unsigned)((total_items + (256 / (DD / 8)) * h3b::kItems - 1) / \
                                           ((256 / (DD / 8)) * h3b::kItems)), 256, 0, stream>>>(   \
      o, (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,        \
      q_row_stride, k_row_stride, v_row_stride, (const __nv_bfloat16*)q_weight,            \
      (const __nv_bfloat16*)k_weight, cos, sin, rows, (int)heads, hl, (int)rotary_dim,     \
      q_eps, k_eps)
  if (head_dim == 64) {
    if (shuffle) H3B_QKP(64, true); else H3B_QKP(64, false);
  } else if (head_dim == 128) {
    if (shuffle) H3B_QKP(128, true); else H3B_QKP(128, false);
  } else {
    if (shuffle) H3B_QKP(256, true); else H3B_QKP(256, false);
  }
#undef H3B_QKP
  return h3b::check_launch("h3b_qknorm_rope_pack");
}

extern "C" int h3b_pack_qkv(void* out, const void* q, const void* k, const void* v,
                            int64_t rows, int64_t heads, int64_t head_dim, int64_t world,
                            int64_t q_row_stride, int64_t q_head_stride, int64_t k_row_stride,
                            int64_t k_head_stride, int64_t v_row_stride,
                            int64_t v_head_stride, h3b_stream_t stream) {
  H3B_REQUIRE(rows >= 0 && heads >= 0 && head_dim >= 0 && world > 0, "pack_qkv: bad shape");
  H3B_REQUIRE(heads % world == 0, "heads (%lld) must divide Ulysses degree (%lld)",
              (long long)heads, (long long)world);
  if (rows == 0 || heads == 0 || head_dim == 0) return H3B_OK;
  const int64_t hl = heads / world;
  auto* o = (__nv_bfloat16*)out;
  auto* qq = (const __nv_bfloat16*)q;
  auto* kk = (const __nv_bfloat16*)k;
  auto* vv = (const __nv_bfloat16*)v;
  const bool vec = (head_dim == 64 || head_dim == 128 || head_dim == 256) && rows <= 0x7fffffffLL &&
                   aligned16(out) && aligned16(q) && aligned16(k) && aligned16(v) &&
                   q_row_stride % 8 == 0 && q_head_stride % 8 == 0 && k_row_stride % 8 == 0 &&
                   k_head_stride % 8 == 0 && v_row_stride % 8 == 0 && v_head_stride % 8 == 0;
  if (vec) {
#define H3B_PK(DD)                                                                       \
  if (head_dim == DD)                                                                    \
    h3b::pack_qkv_kernel<DD><<<(unsigned)rows, 256, 0, stream>>>(                          \
        o, qq, kk, vv, rows, (int)heads, (int)hl, q_row_stride, q_head_stride, k_row_stride, \
        k_head_stride, v_row_stride, v_head_stride);
    H3B_PK(64) H3B_PK(128) H3B_PK(256)
#undef H3B_PK
  } else {
    h3b::pack_qkv_scalar<<<(unsigned)(h3b::num_sms() * 8), 256, 0, stream>>>(
        o, qq, kk, vv, rows, heads, hl, head_dim, q_row_stride, q_head_stride, k_row_stride,
        k_head_stride, v_row_stride, v_head_stride);
  }
  return h3b::check_launch("h3b_pack_qkv");
}

extern "C" int h3b_merge_heads(void* out, const void* x, int64_t world, int64_t rows,
                               int64_t inner, h3b_stream_t stream) {
  H3B_REQUIRE(world >= 0 && rows >= 0 && inner >= 0, "merge_heads: negative shape");
  if (world == 0 || rows == 0 || inner == 0) return H3B_OK;
  auto* o = (__nv_bfloat16*)out;
  auto* xi = (const __nv_bfloat16*)x;
  if (inner % 8 == 0 && aligned16(out) && aligned16(x) && rows <= 0x7fffffffLL) {
    h3b::merge_heads_vec<<<(unsigned)rows, 256, 0, stream>>>(o, xi, world, rows, inner / 8);
  } else {
    h3b::merge_heads_scalar<<<(unsigned)(h3b::num_sms() * 8), 256, 0, stream>>>(o, xi, world,
                                                                               rows, inner);
  }
  return h3b::check_launch("h3b_merge_heads");
}

// Same kernel as the fast path of h3b_qknorm_rope_pack, storing each head row
// into the receive buffer of the rank that owns the head (peer-mapped).
extern "C" int h3b_qknorm_rope_pack_p2p(void* const* recv_ptrs, int64_t world,
                                        int64_t row_offset, int64_t total_rows, const void* q,
                                        const void* k, const void* v, int64_t q_row_stride,
                                        int64_t k_row_stride, int64_t v_row_stride,
                                        const void* q_weight, const void* k_weight,
                                        const float* cos, const float* sin, int64_t rows,
                                        int64_t heads, int64_t head_dim, int64_t rotary_dim,
                                        float q_eps, float k_eps, h3b_stream_t stream) {
  H3B_REQUIRE(rows >= 0 && heads > 0 && world > 0, "qknorm_rope_pack_p2p: bad shape");
  H3B_REQUIRE(world <= h3b::kMaxPeers, "qknorm_rope_pack_p2p: at most %d ranks",
              h3b::kMaxPeers);
  H3B_REQUIRE(heads % world == 0, "heads (%lld) must divide Ulysses degree (%lld)",
              (long long)heads, (long long)world);
  H3B_REQUIRE(rotary_dim >= 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0,
              "fused qknorm+rope requires an even rotary dimension no wider than the head, "
              "got rotary_dim=%lld, head_dim=%lld",
              (long long)rotary_dim, (long long)head_dim);
  if ((head_dim != 64 && head_dim != 128 && head_dim != 256) || rotary_dim % 16 != 0 ||
      (head_dim - rotary_dim) % 16 != 0) {
    h3b::set_error("qknorm_rope_pack_p2p: needs head_dim 64/128/256 and rotary_dim and "
                   "head_dim - rotary_dim multiples of 16");
    return H3B_ERR_UNSUPPORTED;
  }
  H3B_REQUIRE(row_offset >= 0 && rows <= total_rows - row_offset,
              "qknorm_rope_pack_p2p: rows [%lld, %lld) outside the %lld-row receive buffers",
              (long long)row_offset, (long long)(row_offset + rows), (long long)total_rows);
  H3B_REQUIRE(recv_ptrs != nullptr, "qknorm_rope_pack_p2p: null receive pointer array");
  h3b::PeerPtrs ptrs{};
  for (int i = 0; i < world; ++i) {
    ptrs.p[i] = recv_ptrs[i];
    H3B_REQUIRE(ptrs.p[i] != nullptr && aligned16(ptrs.p[i]),
                "qknorm_rope_pack_p2p: receive buffer %d is null or not 16-byte aligned", i);
  }
  if (rows == 0) return H3B_OK;
  H3B_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(q_weight) &&
                  aligned16(k_weight) && q_row_stride % 8 == 0 && k_row_stride % 8 == 0 &&
                  v_row_stride % 8 == 0 &&
                  (rotary_dim == 0 || (aligned16(cos) && aligned16(sin))),
              "qknorm_rope_pack_p2p: tensors must be 16-byte aligned with row strides "
              "divisible by 8");
  const int hl = (int)(heads / world);
  const unsigned grid = (unsigned)((rows + h3b::kTokWarps - 1) / h3b::kTokWarps);
#define H3B_QPP(DD)                                                                         \
  if (head_dim == DD)                                                                       \
    h3b::qknorm_rope_pack_tok<DD><<<grid, h3b::kTokWarps * 32, 0, stream>>>(                  \
        h3b::PeerRecv{ptrs, row_offset, hl}, (const __nv_bfloat16*)q,                       \
        (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, q_row_stride, k_row_stride,     \
        v_row_stride, (const __nv_bfloat16*)q_weight, (const __nv_bfloat16*)k_weight, cos, \
        sin, rows, (int)heads, (int)rotary_dim, q_eps, k_eps);
  H3B_QPP(64) H3B_QPP(128) H3B_QPP(256)
#undef H3B_QPP
  return h3b::check_launch("h3b_qknorm_rope_pack_p2p");
}
