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
// of tokens (32 forward, 64 backward) and slides a W-token window down them;
// the run's tokens are read in blocks (8 tokens forward, 4 backward, whose x
// and dy rows double the loads per block) whose loads are all issued before
// the block's arithmetic and stores (restrict-qualified pointers,
// compile-time dtype), so several loads are in flight per thread at high
// occupancy.  The backward recomputes pre from x, and leaves per-(b, run)
// partial rows of dw in the workspace, summed in a fixed order by a second
// kernel (deterministic).  fp32 arithmetic; outputs in the input dtype, dw in
// the weight dtype.  Block and run sizes chosen by timing at B4 T4096 and
// 3 x 2304 channels: backward 0.439 ms (32-token runs, 8-token blocks) ->
// 0.305 (4-token blocks) -> 0.270 ms (64-token runs).
#include "kdn_common.cuh"

namespace kdn {
namespace {

constexpr int kConvW = 4;
constexpr int kConvRun = 32;      // tokens per thread
constexpr int kConvThreads = 128; // 256 channels per CTA

// Two adjacent channels as one 4-byte (bf16) or 8-byte (fp32) element.
template <bool BF>
using Pair = typename std::conditional<BF, __nv_bfloat162, float2>::type;
template <bool BF>
__device__ __forceinline__ float2 to2(Pair<BF> v) {
  if constexpr (BF) return __bfloat1622float2(v); else return v;
}
template <bool BF>
__device__ __forceinline__ Pair<BF> from2(float a, float b) {
  if constexpr (BF) return __floats2bfloat162_rn(a, b); else return make_float2(a, b);
}
__device__ __forceinline__ float wt(const void* w, size_t i, bool bf) {
  return bf ? __bfloat162float(static_cast<const bf16*>(w)[i]) : static_cast<const float*>(w)[i];
}
// sigmoid with the fast reciprocal (the output is compared at tolerance, not bit for bit)
__device__ __forceinline__ float sig(float p) { return __fdividef(1.f, 1.f + __expf(-p)); }

struct ConvArgs {
  const void* x;
  const void* w;  // [C][W]
  void* y[3];     // forward outputs per group
  const void* dy[3];  // backward cotangents per group (nullable = 0)
  void* dx;
  float* dw_part;  // [B * nruns][C][W]
  int64_t B, T, C, D;
  int w_bf16, silu;
};

constexpr int kConvBlk = 8;   // forward: tokens whose loads are issued together
constexpr int kConvRunB = 64;  // backward: tokens per thread
constexpr int kConvBlkB = 4;   // backward: x and dy rows of 4 tokens per load block (72 registers)
static_assert(kConvBlk >= kConvW - 1 && kConvBlkB >= kConvW - 1, "a load block refills the whole window");

// Per-thread views: row t of this thread's channel pair at p[t * stride]
// (pair units; T * C / 2 < 2^31 is checked on the host).
template <bool XB>
struct ConvRows {
  const Pair<XB>* __restrict__ x;
  unsigned xs;
};

template <bool XB>
__global__ void __launch_bounds__(kConvThreads, 8) short_conv_fwd_kernel(ConvArgs a) {
  const int64_t c = 2 * ((int64_t)blockIdx.x * kConvThreads + threadIdx.x);
  if (c >= a.C) return;
  const int64_t b = blockIdx.z;
  const int t0 = blockIdx.y * kConvRun, t1 = (int)min((int64_t)t0 + kConvRun, a.T);
  const bool wb = a.w_bf16 != 0;
  const int grp = (int)(c / a.D);
  const int64_t cd = c - grp * a.D;
  const Pair<XB>* __restrict__ x = static_cast<const Pair<XB>*>(a.x) + ((size_t)b * a.T * a.C + c) / 2;
  Pair<XB>* __restrict__ y =
      static_cast<Pair<XB>*>(grp == 0 ? a.y[0] : grp == 1 ? a.y[1] : a.y[2]) + ((size_t)b * a.T * a.D + cd) / 2;
  const unsigned xs = (unsigned)(a.C / 2), ys = (unsigned)(a.D / 2);
  float w0[kConvW], w1[kConvW];
#pragma unroll
  for (int j = 0; j < kConvW; ++j) {
    w0[j] = wt(a.w, (size_t)c * kConvW + j, wb);
    w1[j] = wt(a.w, (size_t)(c + 1) * kConvW + j, wb);
  }
  // window of the W-1 tokens before the current block
  float2 h[kConvW - 1];
#pragma unroll
  for (int j = 0; j < kConvW - 1; ++j) {
    const int t = t0 - (kConvW - 1) + j;
    h[j] = t >= 0 ? to2<XB>(x[(unsigned)t * xs]) : make_float2(0.f, 0.f);
  }
#pragma unroll 1
  for (int tb = t0; tb < t1; tb += kConvBlk) {
    float2 v[kConvBlk];
#pragma unroll
    for (int i = 0; i < kConvBlk; ++i)
      v[i] = tb + i < t1 ? to2<XB>(x[(unsigned)(tb + i) * xs]) : make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kConvBlk; ++i) {
      // x[t - W + 1 + j] for j < W - 1 from the window, x[t] = v[i]
      float p0 = w0[kConvW - 1] * v[i].x, p1 = w1[kConvW - 1] * v[i].y;
#pragma unroll
      for (int j = 0; j < kConvW - 1; ++j) {
        const float2 xj = i + j >= kConvW - 1 ? v[i + j - (kConvW - 1)] : h[i + j];
        p0 = fmaf(w0[j], xj.x, p0);
        p1 = fmaf(w1[j], xj.y, p1);
      }
      if (a.silu) {
        p0 *= sig(p0);
        p1 *= sig(p1);
      }
      if (tb + i < t1) y[(unsigned)(tb + i) * ys] = from2<XB>(p0, p1);
    }
#pragma unroll
    for (int j = 0; j < kConvW - 1; ++j) h[j] = v[kConvBlk - (kConvW - 1) + j];
  }
}

template <bool XB>
__global__ void __launch_bounds__(kConvThreads, 6) short_conv_bwd_kernel(ConvArgs a) {
  const int64_t c = 2 * ((int64_t)blockIdx.x * kConvThreads + threadIdx.x);
  if (c >= a.C) return;
  const int64_t b = blockIdx.z;
  const int t0 = blockIdx.y * kConvRunB, t1 = (int)min((int64_t)t0 + kConvRunB, a.T), T = (int)a.T;
  const bool wb = a.w_bf16 != 0;
  const int grp = (int)(c / a.D);
  const int64_t cd = c - grp * a.D;
  const Pair<XB>* __restrict__ x = static_cast<const Pair<XB>*>(a.x) + ((size_t)b * a.T * a.C + c) / 2;
  Pair<XB>* __restrict__ dx = static_cast<Pair<XB>*>(a.dx) + ((size_t)b * a.T * a.C + c) / 2;
  const void* dyv = grp == 0 ? a.dy[0] : grp == 1 ? a.dy[1] : a.dy[2];
  const Pair<XB>* __restrict__ dyg = dyv ? static_cast<const Pair<XB>*>(dyv) + ((size_t)b * a.T * a.D + cd) / 2 : nullptr;
  const unsigned xs = (unsigned)(a.C / 2), ys = (unsigned)(a.D / 2);
  float w0[kConvW], w1[kConvW];
#pragma unroll
  for (int j = 0; j < kConvW; ++j) {
    w0[j] = wt(a.w, (size_t)c * kConvW + j, wb);
    w1[j] = wt(a.w, (size_t)(c + 1) * kConvW + j, wb);
  }
  // s runs over the dpre indices [t0, min(t1 + W - 1, T)) in blocks; the x
  // window holds x[s - W + 1 .. s - 1] and the dpre window dpre[s - W + 1 ..
  // s - 1] (zero before t0: dx of tokens >= t0 needs dpre of tokens >= t0)
  float2 h[kConvW - 1], e[kConvW - 1];
#pragma unroll
  for (int j = 0; j < kConvW - 1; ++j) {
    const int t = t0 - (kConvW - 1) + j;
    h[j] = t >= 0 ? to2<XB>(x[(unsigned)t * xs]) : make_float2(0.f, 0.f);
    e[j] = make_float2(0.f, 0.f);
  }
  float dw0[kConvW], dw1[kConvW];
#pragma unroll
  for (int j = 0; j < kConvW; ++j) dw0[j] = dw1[j] = 0.f;
  const int send = min(t1 + kConvW - 1, T);
#pragma unroll 1
  for (int sb = t0; sb < t1 + kConvW - 1; sb += kConvBlkB) {
    float2 v[kConvBlkB], g[kConvBlkB];
#pragma unroll
    for (int i = 0; i < kConvBlkB; ++i) {
      const bool in = sb + i < send;
      v[i] = in ? to2<XB>(x[(unsigned)(sb + i) * xs]) : make_float2(0.f, 0.f);
      g[i] = in && dyg ? to2<XB>(dyg[(unsigned)(sb + i) * ys]) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < kConvBlkB; ++i) {
      const int s = sb + i;
      float p0 = w0[kConvW - 1] * v[i].x, p1 = w1[kConvW - 1] * v[i].y;
#pragma unroll
      for (int j = 0; j < kConvW - 1; ++j) {
        const float2 xj = i + j >= kConvW - 1 ? v[i + j - (kConvW - 1)] : h[i + j];
        p0 = fmaf(w0[j], xj.x, p0);
        p1 = fmaf(w1[j], xj.y, p1);
      }
      float d0 = g[i].x, d1 = g[i].y;  // dpre[s] (zero at and past the sequence end)
      if (a.silu) {
        const float s0 = sig(p0), s1 = sig(p1);
        d0 *= s0 * (1.f + p0 * (1.f - s0));
        d1 *= s1 * (1.f + p1 * (1.f - s1));
      }
      if (s < t1) {  // dw over the run's own tokens: dpre[s] x[s - W + 1 + j]
#pragma unroll
        for (int j = 0; j < kConvW - 1; ++j) {
          const float2 xj = i + j >= kConvW - 1 ? v[i + j - (kConvW - 1)] : h[i + j];
          dw0[j] = fmaf(d0, xj.x, dw0[j]);
          dw1[j] = fmaf(d1, xj.y, dw1[j]);
        }
        dw0[kConvW - 1] = fmaf(d0, v[i].x, dw0[kConvW - 1]);
        dw1[kConvW - 1] = fmaf(d1, v[i].y, dw1[kConvW - 1]);
      }
      // dx[s - W + 1] = w[0] dpre[s] + sum_{j>=1} w[j] dpre[s - j]
      const int tx = s - (kConvW - 1);
      if (tx >= t0 && tx < t1) {
        float x0 = w0[0] * d0, x1 = w1[0] * d1;
#pragma unroll
        for (int j = 1; j < kConvW; ++j) {
          x0 = fmaf(w0[j], e[kConvW - 1 - j].x, x0);
          x1 = fmaf(w1[j], e[kConvW - 1 - j].y, x1);
        }
        dx[(unsigned)tx * xs] = from2<XB>(x0, x1);
      }
#pragma unroll
      for (int j = 0; j < kConvW - 2; ++j) e[j] = e[j + 1];
      e[kConvW - 2] = make_float2(d0, d1);
    }
#pragma unroll
    for (int j = 0; j < kConvW - 1; ++j) h[j] = v[kConvBlkB - (kConvW - 1) + j];
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
  if (B > 65535 || (T + kConvRunB - 1) / kConvRunB > 65535 || (T + kConvRun - 1) / kConvRun > 65535 ||
      T * C / 2 >= (int64_t)1 << 31)
    return set_error(KDN_ERR_INVALID, "%s: size too large", what);
  return KDN_OK;
}

dim3 conv_grid(int64_t B, int64_t T, int64_t C, int run = kConvRun) {
  return dim3((unsigned)((C / 2 + kConvThreads - 1) / kConvThreads), (unsigned)((T + run - 1) / run),
              (unsigned)B);
}

}  // namespace
}  // namespace kdn

using namespace kdn;

extern "C" {

size_t kdn_short_conv_workspace_bytes(int64_t B, int64_t T, int64_t C, int64_t W) {
  if (B <= 0 || T <= 0 || C <= 0) return 0;
  return align_up(sizeof(float) * (size_t)B * ((T + kConvRunB - 1) / kConvRunB) * C * W, 256);
}

int kdn_short_conv_fwd(const void* x, int x_bf16, const void* weight, int w_bf16, void* const* y, int64_t groups,
                       int64_t B, int64_t T, int64_t C, int64_t W, int silu, kdn_stream_t stream) {
  if (int rc = conv_check("kdn_short_conv_fwd", B, T, C, groups, W)) return rc;
  if (!x || !weight || !y) return set_error(KDN_ERR_INVALID, "kdn_short_conv_fwd: null pointer");
  ConvArgs a{};
  a.x = x; a.w = weight; a.B = B; a.T = T; a.C = C; a.D = C / groups;
  a.w_bf16 = w_bf16; a.silu = silu;
  for (int g = 0; g < groups; ++g) {
    if (!y[g]) return set_error(KDN_ERR_INVALID, "kdn_short_conv_fwd: null output %d", g);
    a.y[g] = y[g];
  }
  if (x_bf16)
    short_conv_fwd_kernel<true><<<conv_grid(B, T, C), kConvThreads, 0, (cudaStream_t)stream>>>(a);
  else
    short_conv_fwd_kernel<false><<<conv_grid(B, T, C), kConvThreads, 0, (cudaStream_t)stream>>>(a);
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
  a.B = B; a.T = T; a.C = C; a.D = C / groups; a.w_bf16 = w_bf16; a.silu = silu;
  for (int g = 0; g < groups; ++g) a.dy[g] = dy[g];
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid = conv_grid(B, T, C, kConvRunB);
  if (x_bf16)
    short_conv_bwd_kernel<true><<<grid, kConvThreads, 0, st>>>(a);
  else
    short_conv_bwd_kernel<false><<<grid, kConvThreads, 0, st>>>(a);
  if (int rc = check_launch("short_conv_bwd_kernel")) return rc;
  const int64_t CW = C * W, nparts = B * grid.y;
  short_conv_dw_kernel<<<(unsigned)((CW + 255) / 256), 256, 0, st>>>(a.dw_part, dweight, nparts, CW, w_bf16);
  return check_launch("short_conv_dw_kernel");
}

}  // extern "C"
