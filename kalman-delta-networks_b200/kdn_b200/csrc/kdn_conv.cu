// Short causal depthwise convolution with SiLU in front of the scan: the
// packed q/k/v convolution of the isotropic mixer (qkv_causal_conv1d,
// lit_gpt/kdn_ops/iso_kdn_chunk.py:459, Function :431, inside PackedQKV :575)
// and the per-tensor one of the diagonal mixer (_fixed_short_conv,
// lit_gpt/diag_kdn.py:75, flash-linear-attention's causal_conv1d).
//
//   pre[b,t,c] = sum_{j<W} w[c,j] x[b, t-W+1+j, c]   (x = 0 before t = 0)
//   y = silu(pre) = pre sigmoid(pre)
// Backward, with dpre = dy silu'(pre), silu'(p) = s (1 + p (1 - s)):
//   dx[t] = sum_j w[c,j] dpre[t+W-1-j],  dw[c,j] = sum_{b,t} dpre[t] x[t-W+1+j]
//
// x is [B,T,C] with channel stride 1; the channels form `groups` blocks of D
// (3 for the packed q|k|v input), each written to / read from its own
// contiguous [B,T,D] tensor.  A thread owns two adjacent channels over a run
// of kConvRun tokens and slides a W-token window down them in registers, so x
// and y move once (plus a three-token halo per run).  The backward recomputes
// pre from x, and leaves per-(b, run) partial rows of dw in the workspace,
// summed in a fixed order by a second kernel (deterministic).  fp32
// arithmetic; outputs in the input dtype, dw in the weight dtype.
#include "kdn_common.cuh"

namespace kdn {
namespace {

constexpr int kConvW = 4;
constexpr int kConvRun = 32;      // tokens per thread
constexpr int kConvThreads = 128; // 256 channels per CTA

__device__ __forceinline__ float2 ld2(const void* p, size_t i, bool bf) {
  if (bf) return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(static_cast<const bf16*>(p) + i));
  return *reinterpret_cast<const float2*>(static_cast<const float*>(p) + i);
}
__device__ __forceinline__ void st2(void* p, size_t i, float a, float b, bool bf) {
  if (bf)
    *reinterpret_cast<__nv_bfloat162*>(static_cast<bf16*>(p) + i) = __floats2bfloat162_rn(a, b);
  else
    *reinterpret_cast<float2*>(static_cast<float*>(p) + i) = make_float2(a, b);
}
__device__ __forceinline__ float wt(const void* w, size_t i, bool bf) {
  return bf ? __bfloat162float(static_cast<const bf16*>(w)[i]) : static_cast<const float*>(w)[i];
}
__device__ __forceinline__ float sig(float p) { return 1.f / (1.f + __expf(-p)); }

struct ConvArgs {
  const void* x;
  const void* w;  // [C][W]
  void* y[3];     // forward outputs per group
  const void* dy[3];  // backward cotangents per group (nullable = 0)
  void* dx;
  float* dw_part;  // [B * nruns][C][W]
  int64_t B, T, C, D;
  int x_bf16, w_bf16, silu;
};

__global__ void __launch_bounds__(kConvThreads) short_conv_fwd_kernel(ConvArgs a) {
  const int64_t c = 2 * ((int64_t)blockIdx.x * kConvThreads + threadIdx.x);
  if (c >= a.C) return;
  const int64_t b = blockIdx.z, t0 = (int64_t)blockIdx.y * kConvRun, t1 = min(t0 + kConvRun, a.T);
  const bool xb = a.x_bf16 != 0, wb = a.w_bf16 != 0;
  const int grp = (int)(c / a.D);
  const int64_t cd = c - grp * a.D;
  float w0[kConvW], w1[kConvW];
#pragma unroll
  for (int j = 0; j < kConvW; ++j) {
    w0[j] = wt(a.w, (size_t)c * kConvW + j, wb);
    w1[j] = wt(a.w, (size_t)(c + 1) * kConvW + j, wb);
  }
  // window of the W-1 tokens before t0
  float h0[kConvW - 1], h1[kConvW - 1];
#pragma unroll
  for (int j = 0; j < kConvW - 1; ++j) {
    const int64_t t = t0 - (kConvW - 1) + j;
    float2 v = make_float2(0.f, 0.f);
    if (t >= 0) v = ld2(a.x, ((size_t)b * a.T + t) * a.C + c, xb);
    h0[j] = v.x;
    h1[j] = v.y;
  }
  for (int64_t t = t0; t < t1; ++t) {
    const float2 v = ld2(a.x, ((size_t)b * a.T + t) * a.C + c, xb);
    float p0 = w0[kConvW - 1] * v.x, p1 = w1[kConvW - 1] * v.y;
#pragma unroll
    for (int j = 0; j < kConvW - 1; ++j) {
      p0 = fmaf(w0[j], h0[j], p0);
      p1 = fmaf(w1[j], h1[j], p1);
    }
#pragma unroll
    for (int j = 0; j < kConvW - 2; ++j) {
      h0[j] = h0[j + 1];
      h1[j] = h1[j + 1];
    }
    h0[kConvW - 2] = v.x;
    h1[kConvW - 2] = v.y;
    if (a.silu) {
      p0 *= sig(p0);
      p1 *= sig(p1);
    }
    st2(a.y[grp], ((size_t)b * a.T + t) * a.D + cd, p0, p1, xb);
  }
}

__global__ void __launch_bounds__(kConvThreads) short_conv_bwd_kernel(ConvArgs a) {
  const int64_t c = 2 * ((int64_t)blockIdx.x * kConvThreads + threadIdx.x);
  if (c >= a.C) return;
  const int64_t b = blockIdx.z, t0 = (int64_t)blockIdx.y * kConvRun, t1 = min(t0 + kConvRun, a.T);
  const bool xb = a.x_bf16 != 0, wb = a.w_bf16 != 0;
  const int grp = (int)(c / a.D);
  const int64_t cd = c - grp * a.D;
  const void* dyg = a.dy[grp];
  float w0[kConvW], w1[kConvW];
#pragma unroll
  for (int j = 0; j < kConvW; ++j) {
    w0[j] = wt(a.w, (size_t)c * kConvW + j, wb);
    w1[j] = wt(a.w, (size_t)(c + 1) * kConvW + j, wb);
  }
  // x[s-W+1 .. s] slides with s; dpre[s-W+1 .. s] too (zero before t0: dx of
  // tokens >= t0 needs dpre of tokens >= t0 only)
  float h0[kConvW - 1], h1[kConvW - 1], e0[kConvW - 1], e1[kConvW - 1];
#pragma unroll
  for (int j = 0; j < kConvW - 1; ++j) {
    const int64_t t = t0 - (kConvW - 1) + j;
    float2 v = make_float2(0.f, 0.f);
    if (t >= 0) v = ld2(a.x, ((size_t)b * a.T + t) * a.C + c, xb);
    h0[j] = v.x;
    h1[j] = v.y;
    e0[j] = e1[j] = 0.f;
  }
  float dw0[kConvW], dw1[kConvW];
#pragma unroll
  for (int j = 0; j < kConvW; ++j) dw0[j] = dw1[j] = 0.f;
  const int64_t send = min(t1 + kConvW - 1, a.T);
  for (int64_t s = t0; s < send; ++s) {
    const size_t row = (size_t)b * a.T + s;
    const float2 v = ld2(a.x, row * a.C + c, xb);
    float p0 = w0[kConvW - 1] * v.x, p1 = w1[kConvW - 1] * v.y;
#pragma unroll
    for (int j = 0; j < kConvW - 1; ++j) {
      p0 = fmaf(w0[j], h0[j], p0);
      p1 = fmaf(w1[j], h1[j], p1);
    }
    float d0 = 0.f, d1 = 0.f;
    if (dyg) {
      const float2 g = ld2(dyg, row * a.D + cd, xb);
      d0 = g.x;
      d1 = g.y;
    }
    if (a.silu) {
      const float s0 = sig(p0), s1 = sig(p1);
      d0 *= s0 * (1.f + p0 * (1.f - s0));
      d1 *= s1 * (1.f + p1 * (1.f - s1));
    }
    if (s < t1) {  // dw over this run's own tokens: dpre[s] x[s-W+1+j]
#pragma unroll
      for (int j = 0; j < kConvW - 1; ++j) {
        dw0[j] = fmaf(d0, h0[j], dw0[j]);
        dw1[j] = fmaf(d1, h1[j], dw1[j]);
      }
      dw0[kConvW - 1] = fmaf(d0, v.x, dw0[kConvW - 1]);
      dw1[kConvW - 1] = fmaf(d1, v.y, dw1[kConvW - 1]);
    }
    // dx[s-W+1] = sum_j w[j] dpre[s-j]
    const int64_t tx = s - (kConvW - 1);
    if (tx >= t0) {
      float x0 = w0[0] * d0, x1 = w1[0] * d1;
#pragma unroll
      for (int j = 1; j < kConvW; ++j) {
        x0 = fmaf(w0[j], e0[kConvW - 1 - j], x0);
        x1 = fmaf(w1[j], e1[kConvW - 1 - j], x1);
      }
      st2(a.dx, ((size_t)b * a.T + tx) * a.C + c, x0, x1, xb);
    }
#pragma unroll
    for (int j = 0; j < kConvW - 2; ++j) {
      h0[j] = h0[j + 1];
      h1[j] = h1[j + 1];
      e0[j] = e0[j + 1];
      e1[j] = e1[j + 1];
    }
    h0[kConvW - 2] = v.x;
    h1[kConvW - 2] = v.y;
    e0[kConvW - 2] = d0;
    e1[kConvW - 2] = d1;
  }
  // tokens of the run whose dx still needs dpre past T (zero): the last W-1
  for (int64_t tx = max(send - (kConvW - 1), t0); tx < t1; ++tx) {
    // dpre[tx .. send-1] are the newest window entries, dpre[>= T] = 0
    float x0 = 0.f, x1 = 0.f;
#pragma unroll
    for (int j = 0; j < kConvW; ++j) {
      const int64_t sj = tx + (kConvW - 1) - j;  // dpre index paired with w[j]
      if (sj < send) {
        const int idx = (int)(sj - (send - (kConvW - 1)));  // position in the window e[0 .. W-2]
        x0 = fmaf(w0[j], e0[idx], x0);
        x1 = fmaf(w1[j], e1[idx], x1);
      }
    }
    st2(a.dx, ((size_t)b * a.T + tx) * a.C + c, x0, x1, xb);
  }
  const size_t part = ((size_t)b * gridDim.y + blockIdx.y) * a.C;
#pragma unroll
  for (int j = 0; j < kConvW; ++j) {
    a.dw_part[(part + c) * kConvW + j] = dw0[j];
    a.dw_part[(part + c + 1) * kConvW + j] = dw1[j];
  }
}

// dw[c][j] = sum over the (b, run) partial rows, in order.
__global__ void short_conv_dw_kernel(const float* __restrict__ part, void* __restrict__ dw, int64_t nparts,
                                     int64_t CW, int w_bf16) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= CW) return;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  int64_t p = 0;
  for (; p + 4 <= nparts; p += 4)
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j] += part[(p + j) * CW + i];
  for (; p < nparts; ++p) s[0] += part[p * CW + i];
  const float v = (s[0] + s[1]) + (s[2] + s[3]);
  if (w_bf16)
    static_cast<bf16*>(dw)[i] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(dw)[i] = v;
}

int conv_check(const char* what, int64_t B, int64_t T, int64_t C, int64_t groups, int64_t W) {
  if (B <= 0 || T <= 0 || groups < 1 || groups > 3 || C <= 0 || C % (2 * groups) != 0 || W != kConvW)
    return set_error(KDN_ERR_INVALID, "%s: B, T > 0, groups in 1..3, C a multiple of 2 * groups, W = 4 required",
                     what);
  if (B > 65535 || (T + kConvRun - 1) / kConvRun > 65535)
    return set_error(KDN_ERR_INVALID, "%s: size too large", what);
  return KDN_OK;
}

dim3 conv_grid(int64_t B, int64_t T, int64_t C) {
  return dim3((unsigned)((C / 2 + kConvThreads - 1) / kConvThreads), (unsigned)((T + kConvRun - 1) / kConvRun),
              (unsigned)B);
}

}  // namespace
}  // namespace kdn

using namespace kdn;

extern "C" {

size_t kdn_short_conv_workspace_bytes(int64_t B, int64_t T, int64_t C, int64_t W) {
  if (B <= 0 || T <= 0 || C <= 0) return 0;
  return align_up(sizeof(float) * (size_t)B * ((T + kConvRun - 1) / kConvRun) * C * W, 256);
}

int kdn_short_conv_fwd(const void* x, int x_bf16, const void* weight, int w_bf16, void* const* y, int64_t groups,
                       int64_t B, int64_t T, int64_t C, int64_t W, int silu, kdn_stream_t stream) {
  if (int rc = conv_check("kdn_short_conv_fwd", B, T, C, groups, W)) return rc;
  if (!x || !weight || !y) return set_error(KDN_ERR_INVALID, "kdn_short_conv_fwd: null pointer");
  ConvArgs a{};
  a.x = x; a.w = weight; a.B = B; a.T = T; a.C = C; a.D = C / groups;
  a.x_bf16 = x_bf16; a.w_bf16 = w_bf16; a.silu = silu;
  for (int g = 0; g < groups; ++g) {
    if (!y[g]) return set_error(KDN_ERR_INVALID, "kdn_short_conv_fwd: null output %d", g);
    a.y[g] = y[g];
  }
  short_conv_fwd_kernel<<<conv_grid(B, T, C), kConvThreads, 0, (cudaStream_t)stream>>>(a);
  return check_launch("short_conv_fwd_kernel");
}

int kdn_short_conv_bwd(const void* x, int x_bf16, const void* weight, int w_bf16, const void* const* dy,
                       int64_t groups, void* dx, void* dweight, int64_t B, int64_t T, int64_t C, int64_t W, int silu,
                       void* workspace, size_t workspace_bytes, kdn_stream_t stream) {
  if (int rc = conv_check("kdn_short_conv_bwd", B, T, C, groups, W)) return rc;
  if (!x || !weight || !dy || !dx || !dweight) return set_error(KDN_ERR_INVALID, "kdn_short_conv_bwd: null pointer");
  if (!workspace || workspace_bytes < kdn_short_conv_workspace_bytes(B, T, C, W))
    return set_error(KDN_ERR_WORKSPACE, "kdn_short_conv_bwd: workspace too small");
  ConvArgs a{};
  a.x = x; a.w = weight; a.dx = dx; a.dw_part = static_cast<float*>(workspace);
  a.B = B; a.T = T; a.C = C; a.D = C / groups; a.x_bf16 = x_bf16; a.w_bf16 = w_bf16; a.silu = silu;
  for (int g = 0; g < groups; ++g) a.dy[g] = dy[g];
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid = conv_grid(B, T, C);
  short_conv_bwd_kernel<<<grid, kConvThreads, 0, st>>>(a);
  if (int rc = check_launch("short_conv_bwd_kernel")) return rc;
  const int64_t CW = C * W, nparts = B * grid.y;
  short_conv_dw_kernel<<<(unsigned)((CW + 255) / 256), 256, 0, st>>>(a.dw_part, dweight, nparts, CW, w_bf16);
  return check_launch("short_conv_dw_kernel");
}

}  // extern "C"
