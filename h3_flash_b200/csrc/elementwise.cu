// AdaLN / norm / activation elementwise kernels of the DiT block.
//
// All are HBM-bound streams: 128-bit loads and stores (ld/st .cs for data
// touched once, __ldg for the small AdaLN tables and norm weights that every
// row re-reads from L2), fp32 math, one round-to-nearest-even bf16 rounding
// per stored value.
//
// Row kernels (the four AdaLN variants) use one warp per row: the row stays in
// registers between the sum-of-squares reduction and the output pass, so each
// activation byte crosses HBM exactly once. NCH = 16-byte chunks per lane.
//
// Semantics follow src/h3_flash/runtime/kernels/fusions.py:23-123 (reference
// Triton kernels) and kernels/transformer.py:72-74, :123-126 (eager ops).
#include <cstdio>

#include "common.cuh"

namespace h3b {
namespace {

enum RowOp : int {
  kRmsModulate = 0,     // out0 = rms(x)*w*(1+scale)+shift
  kResRmsModulate = 1,  // out0 = res+gate*branch ; out1 = rms(out0_fp32)*w*(1+scale)+shift
  kModulate = 2,        // out0 = x*(1+scale)+shift
  kGatedResidual = 3,   // out0 = res+gate*branch
};

struct RowArgs {
  void* out0;
  void* out1;
  const void* in0;
  const void* in1;
  const void* weight;
  const void* gate;
  const void* scale;
  const void* shift;
  const int64_t* index;
  int64_t rows, cols, n_index;
  int64_t in0_stride, in1_stride, out0_stride, out1_stride;
  int64_t gate_stride, scale_stride, shift_stride;
  float eps;
};

constexpr int kRowWarps = 8;

template <int OP, int NCH>
__global__ void __launch_bounds__(kRowWarps * 32) adaln_rows_vec(RowArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int64_t t = a.index[row % a.n_index];
  const int cols = (int)a.cols;

  const __nv_bfloat16* in0 = (const __nv_bfloat16*)a.in0 + row * a.in0_stride;
  const __nv_bfloat16* in1 = (const __nv_bfloat16*)a.in1 + row * a.in1_stride;
  const __nv_bfloat16* gate = (const __nv_bfloat16*)a.gate + t * a.gate_stride;
  const __nv_bfloat16* scale = (const __nv_bfloat16*)a.scale + t * a.scale_stride;
  const __nv_bfloat16* shift = (const __nv_bfloat16*)a.shift + t * a.shift_stride;
  const __nv_bfloat16* weight = (const __nv_bfloat16*)a.weight;

  constexpr bool kTwoIn = (OP == kResRmsModulate || OP == kGatedResidual);
  constexpr bool kNorm = (OP == kRmsModulate || OP == kResRmsModulate);

  // The row stays in registers as packed bf16 (4 registers per 8 values); the
  // fp32 values are recomputed from it where needed instead of being held, so a
  // 3072-wide row costs ~50-100 registers and two CTAs fit per SM.
  uint4 raw0[NCH], raw1[kTwoIn ? NCH : 1];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < cols) {
      raw0[c] = ld_stream(in0 + col);
      if (kTwoIn) raw1[c] = ld_stream(in1 + col);
    }
  }
  auto value = [&](int c, float (&h)[8]) {
    const int col = (c * 32 + lane) * 8;
    f8 x0 = unpack8(raw0[c]);
    if (kTwoIn) {
      f8 x1 = unpack8(raw1[c]);
      f8 g = unpack8(ld_cached(gate + col));
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = x0.v[j] + g.v[j] * x1.v[j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = x0.v[j];
    }
  };

  if (!kNorm) {
    // Streaming ops: one pass, output straight from the loaded chunk.
    __nv_bfloat16* out = (__nv_bfloat16*)a.out0 + row * a.out0_stride;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < cols) {
        float h[8];
        value(c, h);
        if (OP == kModulate) {
          f8 sc = unpack8(ld_cached(scale + col));
          f8 sh = unpack8(ld_cached(shift + col));
#pragma unroll
          for (int j = 0; j < 8; ++j) h[j] = h[j] * (1.f + sc.v[j]) + sh.v[j];
        }
        st_stream(out + col, pack8(h));
      }
    }
    return;
  }

  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < cols) {
      float h[8];
      value(c, h);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += h[j] * h[j];
      if (OP == kResRmsModulate) {
        __nv_bfloat16* out0 = (__nv_bfloat16*)a.out0 + row * a.out0_stride;
        st_stream(out0 + col, pack8(h));
      }
    }
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)cols + a.eps);
  __nv_bfloat16* out =
      (__nv_bfloat16*)(OP == kResRmsModulate ? a.out1 : a.out0) +
      row * (OP == kResRmsModulate ? a.out1_stride : a.out0_stride);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < cols) {
      float h[8];
      value(c, h);
      f8 sc = unpack8(ld_cached(scale + col));
      f8 sh = unpack8(ld_cached(shift + col));
      f8 w = unpack8(ld_cached(weight + col));
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (h[j] * rstd) * w.v[j] * (1.f + sc.v[j]) + sh.v[j];
      st_stream(out + col, pack8(o));
    }
  }
}

// Fallback for shapes the vector kernel cannot address (odd widths, unaligned
// rows): one CTA per row, scalar accesses, the row re-read from L1/L2 for the
// output pass.
template <int OP>
__global__ void __launch_bounds__(256) adaln_rows_scalar(RowArgs a) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const int64_t t = a.index[row % a.n_index];
  const int64_t cols = a.cols;
  const __nv_bfloat16* in0 = (const __nv_bfloat16*)a.in0 + row * a.in0_stride;
  const __nv_bfloat16* in1 = (const __nv_bfloat16*)a.in1 + row * a.in1_stride;
  const __nv_bfloat16* gate = (const __nv_bfloat16*)a.gate + t * a.gate_stride;
  const __nv_bfloat16* scale = (const __nv_bfloat16*)a.scale + t * a.scale_stride;
  const __nv_bfloat16* shift = (const __nv_bfloat16*)a.shift + t * a.shift_stride;
  const __nv_bfloat16* weight = (const __nv_bfloat16*)a.weight;
  constexpr bool kTwoIn = (OP == kResRmsModulate || OP == kGatedResidual);
  constexpr bool kNorm = (OP == kRmsModulate || OP == kResRmsModulate);

  auto value = [&](int64_t c) -> float {
    float x = __bfloat162float(in0[c]);
    if (kTwoIn) x = x + __bfloat162float(gate[c]) * __bfloat162float(in1[c]);
    return x;
  };
  float rstd = 1.f;
  if (kNorm) {
    float ss = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      float x = value(c);
      ss += x * x;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      v = warp_sum(v);
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    rstd = rsqrtf(red[0] / (float)cols + a.eps);
  }
  __nv_bfloat16* out0 = (__nv_bfloat16*)a.out0 + row * a.out0_stride;
  __nv_bfloat16* out1 = (__nv_bfloat16*)a.out1 + row * a.out1_stride;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    float x = value(c);
    if (OP == kGatedResidual) {
      out0[c] = __float2bfloat16_rn(x);
      continue;
    }
    if (OP == kResRmsModulate) out0[c] = __float2bfloat16_rn(x);
    const float sc = __bfloat162float(scale[c]);
    const float sh = __bfloat162float(shift[c]);
    float o;
    if (kNorm)
      o = (x * rstd) * __bfloat162float(weight[c]) * (1.f + sc) + sh;
    else
      o = x * (1.f + sc) + sh;
    if (OP == kResRmsModulate)
      out1[c] = __float2bfloat16_rn(o);
    else
      out0[c] = __float2bfloat16_rn(o);
  }
}

template <int OP, int NCH>
void launch_vec(const RowArgs& a, cudaStream_t s) {
  const unsigned grid = (unsigned)((a.rows + kRowWarps - 1) / kRowWarps);
  adaln_rows_vec<OP, NCH><<<grid, kRowWarps * 32, 0, s>>>(a);
}

template <int OP>
int launch_rows(const RowArgs& a, cudaStream_t s, const char* name) {
  if (a.rows == 0 || a.cols == 0) return H3B_OK;
  constexpr bool kTwoIn = (OP == kResRmsModulate || OP == kGatedResidual);
  constexpr bool kNorm = (OP == kRmsModulate || OP == kResRmsModulate);
  bool vec = (a.cols % 8 == 0) && a.cols <= 24 * 256;
  vec = vec && aligned16(a.in0) && aligned16(a.out0) && a.in0_stride % 8 == 0 &&
        a.out0_stride % 8 == 0 && aligned16(a.scale) && aligned16(a.shift) &&
        a.scale_stride % 8 == 0 && a.shift_stride % 8 == 0;
  if (kTwoIn) vec = vec && aligned16(a.in1) && a.in1_stride % 8 == 0 && aligned16(a.gate) &&
                    a.gate_stride % 8 == 0;
  if (OP == kResRmsModulate) vec = vec && aligned16(a.out1) && a.out1_stride % 8 == 0;
  if (kNorm) vec = vec && aligned16(a.weight);
  if (vec) {
    const int nch = (int)((a.cols + 255) / 256);
    switch (nch) {
#define H3B_CASE(N) \
  case N:           \
    launch_vec<OP, N>(a, s); \
    break;
      H3B_CASE(1) H3B_CASE(2) H3B_CASE(3) H3B_CASE(4) H3B_CASE(5) H3B_CASE(6)
      H3B_CASE(7) H3B_CASE(8) H3B_CASE(9) H3B_CASE(10) H3B_CASE(11) H3B_CASE(12)
      H3B_CASE(13) H3B_CASE(14) H3B_CASE(15) H3B_CASE(16) H3B_CASE(17) H3B_CASE(18)
      H3B_CASE(19) H3B_CASE(20) H3B_CASE(21) H3B_CASE(22) H3B_CASE(23) H3B_CASE(24)
#undef H3B_CASE
      default:
        break;
    }
  } else {
    H3B_REQUIRE(a.rows <= 0x7fffffffLL, "%s: too many rows (%lld)", name, (long long)a.rows);
    adaln_rows_scalar<OP><<<(unsigned)a.rows, 256, 0, s>>>(a);
  }
  return check_launch(name);
}

// ---- SwiGLU and GELU-tanh -------------------------------------------------

constexpr int kEwThreads = 256;
constexpr int kEwUnroll = 4;

// One CTA walks rows (grid-stride); threads walk 16-byte chunks of a row,
// kEwUnroll chunks in flight per thread.
template <bool kSwiglu>
__global__ void __launch_bounds__(kEwThreads) act_rows_vec(void* out, const void* x, int64_t rows,
                                                          int64_t n, int64_t in_stride,
                                                          int64_t out_stride) {
  const int64_t n8 = n / 8;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* xr = (const __nv_bfloat16*)x + r * in_stride;
    __nv_bfloat16* orow = (__nv_bfloat16*)out + r * out_stride;
    for (int64_t base = threadIdx.x; base < n8; base += (int64_t)kEwThreads * kEwUnroll) {
      uint4 va[kEwUnroll], vg[kEwUnroll];
#pragma unroll
      for (int u = 0; u < kEwUnroll; ++u) {
        const int64_t c = base + (int64_t)u * kEwThreads;
        if (c < n8) {
          va[u] = ld_stream(xr + c * 8);
          if (kSwiglu) vg[u] = ld_stream(xr + n + c * 8);
        }
      }
#pragma unroll
      for (int u = 0; u < kEwUnroll; ++u) {
        const int64_t c = base + (int64_t)u * kEwThreads;
        if (c < n8) {
          f8 a = unpack8(va[u]);
          float o[8];
          if (kSwiglu) {
            f8 g = unpack8(vg[u]);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = a.v[j] * silu(g.v[j]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = gelu_tanh(a.v[j]);
          }
          st_stream(orow + c * 8, pack8(o));
        }
      }
    }
  }
}

template <bool kSwiglu>
__global__ void __launch_bounds__(kEwThreads) act_rows_scalar(void* out, const void* x,
                                                             int64_t rows, int64_t n,
                                                             int64_t in_stride,
                                                             int64_t out_stride) {
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* xr = (const __nv_bfloat16*)x + r * in_stride;
    __nv_bfloat16* orow = (__nv_bfloat16*)out + r * out_stride;
    for (int64_t c = threadIdx.x; c < n; c += kEwThreads) {
      const float a = __bfloat162float(xr[c]);
      float o;
      if (kSwiglu)
        o = a * silu(__bfloat162float(xr[n + c]));
      else
        o = gelu_tanh(a);
      orow[c] = __float2bfloat16_rn(o);
    }
  }
}

template <bool kSwiglu>
int launch_act(void* out, const void* x, int64_t rows, int64_t n, int64_t in_stride,
               int64_t out_stride, cudaStream_t s, const char* name) {
  if (rows == 0 || n == 0) return H3B_OK;
  const int64_t max_grid = (int64_t)num_sms() * 16;
  const unsigned grid = (unsigned)(rows < max_grid ? rows : max_grid);
  const bool vec = n % 8 == 0 && aligned16(x) && aligned16(out) && in_stride % 8 == 0 &&
                   out_stride % 8 == 0;
  if (vec)
    act_rows_vec<kSwiglu><<<grid, kEwThreads, 0, s>>>(out, x, rows, n, in_stride, out_stride);
  else
    act_rows_scalar<kSwiglu><<<grid, kEwThreads, 0, s>>>(out, x, rows, n, in_stride, out_stride);
  return check_launch(name);
}

}  // namespace
}  // namespace h3b

using h3b::RowArgs;

extern "C" int h3b_rmsnorm_modulate(void* out, const void* x, const void* weight,
                                    const void* scale, const void* shift,
                                    const int64_t* index, int64_t rows, int64_t cols,
                                    int64_t n_index, int64_t x_row_stride,
                                    int64_t out_row_stride, int64_t scale_row_stride,
                                    int64_t shift_row_stride, float eps,
                                    h3b_stream_t stream) {
  H3B_REQUIRE(rows >= 0 && cols >= 0, "rmsnorm_modulate: negative shape");
  H3B_REQUIRE(rows == 0 || n_index > 0, "rmsnorm_modulate: empty index");
  RowArgs a{};
  a.out0 = out;
  a.in0 = x;
  a.weight = weight;
  a.scale = scale;
  a.shift = shift;
  a.gate = scale;
  a.in1 = x;
  a.index = index;
  a.rows = rows;
  a.cols = cols;
  a.n_index = n_index;
  a.in0_stride = x_row_stride;
  a.out0_stride = out_row_stride;
  a.scale_stride = scale_row_stride;
  a.shift_stride = shift_row_stride;
  a.eps = eps;
  return h3b::launch_rows<h3b::kRmsModulate>(a, stream, "h3b_rmsnorm_modulate");
}

extern "C" int h3b_residual_gate_rmsnorm_modulate(
    void* hidden_out, void* normed_out, const void* residual, const void* branch,
    const void* weight, const void* gate, const void* scale, const void* shift,
    const int64_t* index, int64_t rows, int64_t cols, int64_t n_index, int64_t row_stride,
    int64_t gate_row_stride, int64_t scale_row_stride, int64_t shift_row_stride, float eps,
    h3b_stream_t stream) {
  H3B_REQUIRE(rows >= 0 && cols >= 0, "residual_gate_rmsnorm_modulate: negative shape");
  H3B_REQUIRE(rows == 0 || n_index > 0, "residual_gate_rmsnorm_modulate: empty index");
  RowArgs a{};
  a.out0 = hidden_out;
  a.out1 = normed_out;
  a.in0 = residual;
  a.in1 = branch;
  a.weight = weight;
  a.gate = gate;
  a.scale = scale;
  a.shift = shift;
  a.index = index;
  a.rows = rows;
  a.cols = cols;
  a.n_index = n_index;
  a.in0_stride = a.in1_stride = a.out0_stride = a.out1_stride = row_stride;
  a.gate_stride = gate_row_stride;
  a.scale_stride = scale_row_stride;
  a.shift_stride = shift_row_stride;
  a.eps = eps;
  return h3b::launch_rows<h3b::kResRmsModulate>(a, stream,
                                                "h3b_residual_gate_rmsnorm_modulate");
}

extern "C" int h3b_modulate(void* out, const void* x, const void* scale, const void* shift,
                            const int64_t* index, int64_t rows, int64_t cols,
                            int64_t n_index, int64_t x_row_stride, int64_t out_row_stride,
                            int64_t scale_row_stride, int64_t shift_row_stride,
                            h3b_stream_t stream) {
  H3B_REQUIRE(rows >= 0 && cols >= 0, "modulate: negative shape");
  H3B_REQUIRE(rows == 0 || n_index > 0, "modulate: empty index");
  RowArgs a{};
  a.out0 = out;
  a.in0 = x;
  a.in1 = x;
  a.weight = scale;
  a.gate = scale;
  a.scale = scale;
  a.shift = shift;
  a.index = index;
  a.rows = rows;
  a.cols = cols;
  a.n_index = n_index;
  a.in0_stride = x_row_stride;
  a.out0_stride = out_row_stride;
  a.scale_stride = scale_row_stride;
  a.shift_stride = shift_row_stride;
  return h3b::launch_rows<h3b::kModulate>(a, stream, "h3b_modulate");
}

extern "C" int h3b_gated_residual(void* out, const void* residual, const void* branch,
                                  const void* gate, const int64_t* index, int64_t rows,
                                  int64_t cols, int64_t n_index, int64_t row_stride,
                                  int64_t gate_row_stride, h3b_stream_t stream) {
  H3B_REQUIRE(rows >= 0 && cols >= 0, "gated_residual: negative shape");
  H3B_REQUIRE(rows == 0 || n_index > 0, "gated_residual: empty index");
  RowArgs a{};
  a.out0 = out;
  a.in0 = residual;
  a.in1 = branch;
  a.gate = gate;
  a.scale = gate;
  a.shift = gate;
  a.weight = gate;
  a.index = index;
  a.rows = rows;
  a.cols = cols;
  a.n_index = n_index;
  a.in0_stride = a.in1_stride = a.out0_stride = row_stride;
  a.gate_stride = a.scale_stride = a.shift_stride = gate_row_stride;
  return h3b::launch_rows<h3b::kGatedResidual>(a, stream, "h3b_gated_residual");
}

extern "C" int h3b_swiglu(void* out, const void* x, int64_t rows, int64_t n,
                          int64_t in_row_stride, int64_t out_row_stride,
                          h3b_stream_t stream) {
  H3B_REQUIRE(rows >= 0 && n >= 0, "swiglu: negative shape");
  return h3b::launch_act<true>(out, x, rows, n, in_row_stride, out_row_stride, stream,
                               "h3b_swiglu");
}

extern "C" int h3b_gelu_tanh(void* out, const void* x, int64_t rows, int64_t cols,
                             int64_t in_row_stride, int64_t out_row_stride,
                             h3b_stream_t stream) {
  H3B_REQUIRE(rows >= 0 && cols >= 0, "gelu_tanh: negative shape");
  return h3b::launch_act<false>(out, x, rows, cols, in_row_stride, out_row_stride, stream,
                                "h3b_gelu_tanh");
}
