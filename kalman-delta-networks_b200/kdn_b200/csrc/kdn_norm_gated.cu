// Gated RMS normalisation of the scan output (the mixers' o_norm,
// lit_gpt/iso_kdn.py:192-197, 305-314 and lit_gpt/diag_kdn.py:216-221,
// 346-355: flash-linear-attention's FusedRMSNormGated, activation "sigmoid",
// per head row of D = head_v_dim).
//
// Forward, per row x (D values) with gate g and weight w:
//   rstd = 1 / sqrt(mean(x^2) + eps),  y = (x rstd) w act(g)
// with act(g) = sigmoid(g) or g sigmoid(g) ("swish"); rstd is saved.
// Backward, with s = sigmoid(g), xh = x rstd, y0 = xh w:
//   dg = dy y0 s (1 - s)               (sigmoid)   dy' = dy s
//   dg = dy y0 (s + g s (1 - s))       (swish)     dy' = dy g s
//   dw = sum over rows of dy' xh,  c = mean(xh dy' w),  dx = (dy' w - xh c) rstd
// (the published algorithm of fla.modules.fused_norm_gate, installed 0.5.1;
// the reference pins flash-linear-attention at commit 4b02d15).
//
// One warp per row, D / 32 consecutive values per lane (one 4- or 8-byte
// access per tensor and lane, every row one coalesced run); fp32 arithmetic.
// The weight gradient leaves per-CTA partial rows in the workspace, summed
// over CTAs in a fixed order by a second kernel (deterministic).
#include "kdn_common.cuh"

namespace kdn {
namespace {

constexpr int kNgWarps = 8;
constexpr int kNgMaxCtas = 148 * 8;  // eight resident 256-thread CTAs per SM

template <int V>
__device__ __forceinline__ void ld_vec(float (&d)[V], const void* p, size_t off, bool bf) {
  if (bf) {
    const bf16* q = static_cast<const bf16*>(p) + off;
    if constexpr (V == 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(q);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
      const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
      d[0] = a.x; d[1] = a.y; d[2] = b.x; d[3] = b.y;
    } else {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(q));
      d[0] = a.x; d[1] = a.y;
    }
  } else {
    const float* q = static_cast<const float*>(p) + off;
    if constexpr (V == 4) {
      const float4 a = *reinterpret_cast<const float4*>(q);
      d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w;
    } else {
      const float2 a = *reinterpret_cast<const float2*>(q);
      d[0] = a.x; d[1] = a.y;
    }
  }
}

template <int V>
__device__ __forceinline__ void st_vec(void* p, size_t off, const float (&s)[V], bool bf) {
  if (bf) {
    bf16* q = static_cast<bf16*>(p) + off;
    if constexpr (V == 4) {
      uint2 u;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
      h[0] = __floats2bfloat162_rn(s[0], s[1]);
      h[1] = __floats2bfloat162_rn(s[2], s[3]);
      *reinterpret_cast<uint2*>(q) = u;
    } else {
      *reinterpret_cast<__nv_bfloat162*>(q) = __floats2bfloat162_rn(s[0], s[1]);
    }
  } else {
    float* q = static_cast<float*>(p) + off;
    if constexpr (V == 4)
      *reinterpret_cast<float4*>(q) = make_float4(s[0], s[1], s[2], s[3]);
    else
      *reinterpret_cast<float2*>(q) = make_float2(s[0], s[1]);
  }
}

// sigmoid with the fast reciprocal (the output is compared at tolerance, not bit for bit)
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

struct NgArgs {
  const void* x;
  const void* g;
  const float* w;
  void* y;
  float* rstd;
  const void* dy;
  void* dx;
  void* dg;
  float* dw_part;  // [gridDim.x][D]
  int64_t rows;
  float eps;
  int x_bf16, g_bf16, swish;
};

// Each warp takes several rows per iteration and requests all of their
// inputs before any arithmetic (more loads in flight per warp).  Chosen by
// timing at B4 T4096 H18 (bf16): forward 4 rows (0.052 -> 0.045 ms against 2
// rows); backward 2 rows at four 256-thread CTAs per SM (64 registers: 0.177
// -> 0.152 ms; 4 rows or one row at six CTAs per SM were slower).
constexpr int kNgRows = 2;   // backward (and the launch grid)
constexpr int kNgRowsF = 4;  // forward

template <int D>
__global__ void __launch_bounds__(32 * kNgWarps) rmsnorm_gated_fwd_kernel(NgArgs a) {
  constexpr int V = D / 32, R = kNgRowsF;
  const int lane = threadIdx.x & 31;
  const bool xb = a.x_bf16 != 0, gb = a.g_bf16 != 0;
  float w[V];
#pragma unroll
  for (int i = 0; i < V; ++i) w[i] = a.w ? a.w[V * lane + i] : 1.f;
  const int64_t step = (int64_t)gridDim.x * kNgWarps * R;
  for (int64_t row0 = ((int64_t)blockIdx.x * kNgWarps + (threadIdx.x >> 5)) * R; row0 < a.rows; row0 += step) {
    float x[R][V], g[R][V];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (row0 + r < a.rows) {
        const size_t off = (size_t)(row0 + r) * D + V * lane;
        ld_vec<V>(x[r], a.x, off, xb);
        ld_vec<V>(g[r], a.g, off, gb);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) x[r][i] = g[r][i] = 0.f;
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (row0 + r >= a.rows) break;
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) ss = fmaf(x[r][i], x[r][i], ss);
      ss = warp_sum(ss);
      const float rstd = rsqrtf(ss * (1.f / (float)D) + a.eps);
      float y[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float sg = sigmoid_f(g[r][i]);
        y[i] = x[r][i] * rstd * w[i] * (a.swish ? g[r][i] * sg : sg);
      }
      st_vec<V>(a.y, (size_t)(row0 + r) * D + V * lane, y, xb);
      if (lane == 0) a.rstd[row0 + r] = rstd;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(32 * kNgWarps, 4) rmsnorm_gated_bwd_kernel(NgArgs a) {
  constexpr int V = D / 32, R = kNgRows;
  __shared__ float red[kNgWarps][D];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool xb = a.x_bf16 != 0, gb = a.g_bf16 != 0;
  float w[V], dw[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    w[i] = a.w ? a.w[V * lane + i] : 1.f;
    dw[i] = 0.f;
  }
  const int64_t step = (int64_t)gridDim.x * kNgWarps * R;
  for (int64_t row0 = ((int64_t)blockIdx.x * kNgWarps + warp) * R; row0 < a.rows; row0 += step) {
    float x[R][V], g[R][V], dy[R][V], rs[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (row0 + r < a.rows) {
        const size_t off = (size_t)(row0 + r) * D + V * lane;
        ld_vec<V>(x[r], a.x, off, xb);
        ld_vec<V>(g[r], a.g, off, gb);
        ld_vec<V>(dy[r], a.dy, off, xb);  // the output (and its cotangent) has x's dtype
        rs[r] = a.rstd[row0 + r];
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) x[r][i] = g[r][i] = dy[r][i] = 0.f;
        rs[r] = 0.f;
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (row0 + r >= a.rows) break;
      const float rstd = rs[r];
      float dgo[V], wdy[V], xh[V], c = 0.f;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float sg = sigmoid_f(g[r][i]);
        xh[i] = x[r][i] * rstd;
        const float y0 = xh[i] * w[i];
        float d;
        if (a.swish) {
          dgo[i] = dy[r][i] * y0 * (sg + g[r][i] * sg * (1.f - sg));
          d = dy[r][i] * g[r][i] * sg;
        } else {
          dgo[i] = dy[r][i] * y0 * sg * (1.f - sg);
          d = dy[r][i] * sg;
        }
        dw[i] = fmaf(d, xh[i], dw[i]);
        wdy[i] = d * w[i];
        c = fmaf(xh[i], wdy[i], c);
      }
      c = warp_sum(c) * (1.f / (float)D);
      float dxo[V];
#pragma unroll
      for (int i = 0; i < V; ++i) dxo[i] = (wdy[i] - xh[i] * c) * rstd;
      const size_t off = (size_t)(row0 + r) * D + V * lane;
      st_vec<V>(a.dx, off, dxo, xb);
      st_vec<V>(a.dg, off, dgo, gb);
    }
  }
  if (a.dw_part) {
#pragma unroll
    for (int i = 0; i < V; ++i) red[warp][V * lane + i] = dw[i];
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < kNgWarps; ++k) sum += red[k][d];
      a.dw_part[(size_t)blockIdx.x * D + d] = sum;
    }
  }
}

// dweight[d] = sum over CTAs of the partial rows, in CTA order.
__global__ void rmsnorm_gated_dw_kernel(const float* __restrict__ part, float* __restrict__ dw, int nparts, int D) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float s[4] = {0.f, 0.f, 0.f, 0.f};  // four independent chains, combined in a fixed order
  int p = 0;
  for (; p + 4 <= nparts; p += 4)
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j] += part[(size_t)(p + j) * D + d];
  for (; p < nparts; ++p) s[0] += part[(size_t)p * D + d];
  dw[d] = (s[0] + s[1]) + (s[2] + s[3]);
}

unsigned ng_grid(int64_t rows) {
  const int64_t blocks = (rows + kNgWarps * kNgRows - 1) / (kNgWarps * kNgRows);
  return (unsigned)(blocks < kNgMaxCtas ? (blocks > 0 ? blocks : 1) : kNgMaxCtas);
}

int ng_check(const char* what, int64_t rows, int64_t D, int activation) {
  if (rows < 0 || (D != 64 && D != 128))
    return set_error(KDN_ERR_INVALID, "%s: rows >= 0 and D in {64, 128} required", what);
  if (activation != 0 && activation != 1)
    return set_error(KDN_ERR_INVALID, "%s: activation must be 0 (sigmoid) or 1 (swish)", what);
  return KDN_OK;
}

}  // namespace
}  // namespace kdn

using namespace kdn;

extern "C" {

size_t kdn_rmsnorm_gated_workspace_bytes(int64_t rows, int64_t D) {
  return align_up(sizeof(float) * (size_t)ng_grid(rows) * (size_t)(D > 0 ? D : 0), 256);
}

int kdn_rmsnorm_gated_fwd(const void* x, int x_bf16, const void* g, int g_bf16, const float* weight, void* y,
                          float* rstd, int64_t rows, int64_t D, float eps, int activation, kdn_stream_t stream) {
  if (int rc = ng_check("kdn_rmsnorm_gated_fwd", rows, D, activation)) return rc;
  if (rows == 0) return KDN_OK;
  if (!x || !g || !y || !rstd) return set_error(KDN_ERR_INVALID, "kdn_rmsnorm_gated_fwd: null pointer");
  NgArgs a{};
  a.x = x; a.g = g; a.w = weight; a.y = y; a.rstd = rstd; a.rows = rows; a.eps = eps;
  a.x_bf16 = x_bf16; a.g_bf16 = g_bf16; a.swish = activation;
  cudaStream_t st = (cudaStream_t)stream;
  if (D == 128)
    rmsnorm_gated_fwd_kernel<128><<<ng_grid(rows), 32 * kNgWarps, 0, st>>>(a);
  else
    rmsnorm_gated_fwd_kernel<64><<<ng_grid(rows), 32 * kNgWarps, 0, st>>>(a);
  return check_launch("rmsnorm_gated_fwd_kernel");
}

int kdn_rmsnorm_gated_bwd(const void* x, int x_bf16, const void* g, int g_bf16, const float* weight, const void* dy,
                          const float* rstd, void* dx, void* dg, float* dweight, int64_t rows, int64_t D,
                          int activation, void* workspace, size_t workspace_bytes, kdn_stream_t stream) {
  if (int rc = ng_check("kdn_rmsnorm_gated_bwd", rows, D, activation)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (rows == 0) {
    if (dweight && cudaMemsetAsync(dweight, 0, sizeof(float) * D, st) != cudaSuccess)
      return check_launch("memset dweight");
    return KDN_OK;
  }
  if (!x || !g || !dy || !rstd || !dx || !dg) return set_error(KDN_ERR_INVALID, "kdn_rmsnorm_gated_bwd: null pointer");
  if (dweight && (!workspace || workspace_bytes < kdn_rmsnorm_gated_workspace_bytes(rows, D)))
    return set_error(KDN_ERR_WORKSPACE, "kdn_rmsnorm_gated_bwd: workspace too small");
  NgArgs a{};
  a.x = x; a.g = g; a.w = weight; a.dy = dy; a.rstd = const_cast<float*>(rstd); a.dx = dx; a.dg = dg;
  a.dw_part = dweight ? static_cast<float*>(workspace) : nullptr;
  a.rows = rows; a.x_bf16 = x_bf16; a.g_bf16 = g_bf16; a.swish = activation;
  const unsigned grid = ng_grid(rows);
  if (D == 128)
    rmsnorm_gated_bwd_kernel<128><<<grid, 32 * kNgWarps, 0, st>>>(a);
  else
    rmsnorm_gated_bwd_kernel<64><<<grid, 32 * kNgWarps, 0, st>>>(a);
  if (int rc = check_launch("rmsnorm_gated_bwd_kernel")) return rc;
  if (!dweight) return KDN_OK;
  rmsnorm_gated_dw_kernel<<<1, (unsigned)D, 0, st>>>(a.dw_part, dweight, (int)grid, (int)D);
  return check_launch("rmsnorm_gated_dw_kernel");
}

}  // extern "C"
