// Isotropic gate frontend: the per-token scalar preparation in front of the
// covariance ("gain") scan and the memory scan.  Replaces the launches behind
// _iso_kdn_gate_precumsum_paired (lit_gpt/kdn_ops/iso_kdn_chunk.py:1396), i.e.
// _iso_kdn_gate_precumsum_fwd_kernel (740-814), _iso_kdn_gate_precumsum_bwd_kernel
// (817-953) and the three partial-sum reductions (956-1009).
//
// Forward, for token t of stream (b, h) and key channel k:
//   x = g_raw + dt_bias[h, k],  g = -exp(A_log[h]) softplus(x)
//   g_cumsum = log2(e) * (inclusive prefix of g over the 64-token chunk)
//   a = mean_k exp(2 g),  omega = omega_min + softplus(omega_raw + omega_bias[h])
//   r = r_min + softplus(r_raw + r_bias[h]),  initial_precision = 0.1 + softplus(param[h])
// where omega_raw, r_raw are the two halves of the last dimension of
// omega_r_raw [B, T, 2H].  softplus(x) = x above 20, else ln(1 + e^x): the
// definition of flash-linear-attention 0.5.1 (fla/ops/utils/softplus.py),
// which the reference calls and evaluates with the hardware base-2
// exponential and logarithm, as here.
//
// Backward, with dg_pre the memory scan's gate cotangent (natural-log
// coordinates, before the reverse prefix sum):
//   dg = reverse prefix of dg_pre over the chunk + da (2 / K) exp(2 g)
//   dg_raw = dg (-exp(A_log)) sigmoid(x);  dA_log = sum dg g;  ddt_bias = sum_{b,t} dg_raw
//   domega_raw = domega sigmoid(omega_raw + omega_bias) (dr_raw alike), their
//   sums over (b, t) for the biases;  d_param = d_initial_precision sigmoid(param)
// The sums over (b, t) go through per-CTA partials and one reduction kernel
// (a fixed order, so the result is deterministic).
//
// One CTA per (batch, 64-token chunk, head), heads fastest in the grid, and a
// pair of adjacent key channels per thread (K / 2 threads): token rows are
// contiguous over channels, so each token is one coalesced row load / store
// per CTA, and the chunk prefix (reverse prefix in the backward) runs down
// each thread's own two channels.  The per-token channel mean uses a warp
// transpose-reduce.  Every frontend kernel is compiled for 2048 / K resident
// CTAs per SM (32 warps at K = 128) and loads 8-16 tokens per pass: more
// loads in flight per SM than 8 CTAs with twice the tokens per pass, which
// measured 25% slower in the backward.
#include "kdn_common.cuh"

namespace kdn {
namespace {

constexpr int kGateChunk = 64;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float softplus_fla(float x) {
  return x > 20.f ? x : kLn2 * __log2f(1.f + ex2a(x * kLog2e));
}
__device__ __forceinline__ float sigmoid_(float x) { return 1.f / (1.f + expf(-x)); }

__device__ __forceinline__ float ld_any(const void* p, size_t i, bool bf) {
  return bf ? __bfloat162float(static_cast<const bf16*>(p)[i]) : static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_any(void* p, size_t i, bool bf, float v) {
  if (bf) {
    static_cast<bf16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    static_cast<float*>(p)[i] = v;
  }
}

struct GateArgs {
  const void* g_raw;
  const void* omega_r_raw;
  const float *omega_bias, *r_bias, *A_log, *dt_bias, *param;
  long long stride_b, stride_t;  // omega_r_raw strides (elements); the last one is 1
  int T, H, NT;
  bool g_bf16, wr_bf16;
};

// A pair of adjacent channels per thread: one 4- or 8-byte load and store
// per token and thread, K / 2 threads per CTA.
__device__ __forceinline__ float2 ld2(const bf16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
__device__ __forceinline__ float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }

// g = -exp(A_log) softplus(x), with negA = -exp(A_log)
__device__ __forceinline__ float gate_of(float x, float negA) {
  return x > 20.f ? negA * x : (negA * kLn2) * __log2f(1.f + ex2a(x * kLog2e));
}

template <int K, class GT>
__global__ void __launch_bounds__(K / 2, 2048 / K) iso_gate_fwd_kernel(GateArgs g, float omega_min, float r_min,
                                                                       float* __restrict__ g_cumsum,
                                                                       float* __restrict__ a,
                                                                       float* __restrict__ omega,
                                                                       float* __restrict__ r,
                                                                       float* __restrict__ init_prec) {
  constexpr int C = kGateChunk, N = 16, NTH = K / 2, NW = NTH / 32;
  __shared__ float red[NW * N];
  const int bc = blockIdx.x / g.H, h = blockIdx.x - bc * g.H, tid = threadIdx.x, k0 = 2 * tid;
  const int lane = tid & 31, warp = tid >> 5;
  const int b = g.NT ? bc / g.NT : 0, c = g.NT ? bc - b * g.NT : 0;
  const int t0 = c * C, n = min(C, g.T - t0);
  const size_t row0 = ((size_t)b * g.T + t0) * g.H + h;  // row of token t0, in K-vectors
  const size_t rs = (size_t)g.H * K;                       // elements between consecutive tokens
  if (n > 0) {
    const float negA = -expf(g.A_log[h]);
    const float2 bias = ld2(g.dt_bias + (size_t)h * K + k0);
    const GT* src = static_cast<const GT*>(g.g_raw) + row0 * K + k0;
    float* dst = g_cumsum + row0 * K + k0;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 1
    for (int j0 = 0; j0 < C; j0 += N) {
      float2 x[N];
      const GT* p = src + (size_t)j0 * rs;
#pragma unroll
      for (int j = 0; j < N; ++j, p += rs) x[j] = j0 + j < n ? ld2(p) : make_float2(0.f, 0.f);
      float al[N];
      float* q = dst + (size_t)j0 * rs;
#pragma unroll
      for (int j = 0; j < N; ++j, q += rs) {
        al[j] = 0.f;
        if (j0 + j < n) {
          const float g0 = gate_of(x[j].x + bias.x, negA), g1 = gate_of(x[j].y + bias.y, negA);
          s0 += g0;
          s1 += g1;
          st_pair(q, s0 * kLog2e, s1 * kLog2e);
          al[j] = ex2a(2.f * kLog2e * g0) + ex2a(2.f * kLog2e * g1);
        }
      }
      // a = channel mean of exp(2 g): lane j of each warp sums token j0 + j
      static_assert(N <= 32, "one token per lane");
      const float ws = transpose_reduce<N>(al);
      if (lane < N) red[warp * N + lane] = ws;  // lanes >= N repeat lane % N
      __syncthreads();
      if (tid < N && j0 + tid < n) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) sum += red[w * N + tid];
        a[row0 + (size_t)(j0 + tid) * g.H] = sum / (float)K;
      }
      __syncthreads();
    }
    // omega, r: one token per thread
    for (int t = tid; t < n; t += NTH) {
      const size_t o = (size_t)b * g.stride_b + (size_t)(t0 + t) * g.stride_t + h;
      const float wr = ld_any(g.omega_r_raw, o, g.wr_bf16) + g.omega_bias[h];
      const float rr = ld_any(g.omega_r_raw, o + g.H, g.wr_bf16) + g.r_bias[h];
      omega[row0 + (size_t)t * g.H] = omega_min + softplus_fla(wr);
      r[row0 + (size_t)t * g.H] = r_min + softplus_fla(rr);
    }
  }
  if (bc == 0 && tid == 0) init_prec[h] = 0.1f + softplus_fla(g.param[h]);
}

struct GateGrads {
  const float *dg_pre, *da, *domega, *dr, *d_init;  // nullable cotangents
  void* dg_raw;                                      // g_raw's dtype, nullable
  void* domega_r_raw;                                // omega_r_raw's dtype [B, T, 2H], nullable
  float* part_wr;                                    // [NP][2H] or null
  float* part_A;                                     // [NP][H] or null
  float* part_dt;                                    // [NP][H][K] or null
  float* d_param;                                    // [H] or null
};

template <int K, class GT>
__global__ void __launch_bounds__(K / 2, 2048 / K) iso_gate_bwd_kernel(GateArgs g, GateGrads d) {
  constexpr int C = kGateChunk, N = 8, NTH = K / 2, NW = NTH / 32;
  __shared__ float red[NW * 3];
  const int bc = blockIdx.x / g.H, h = blockIdx.x - bc * g.H, tid = threadIdx.x, k0 = 2 * tid;
  const int warp = tid >> 5, lane = tid & 31;
  const int b = g.NT ? bc / g.NT : 0, c = g.NT ? bc - b * g.NT : 0;
  const int t0 = c * C, n = min(C, g.T - t0);
  const size_t row0 = ((size_t)b * g.T + t0) * g.H + h;
  const size_t rs = (size_t)g.H * K;
  const bool need_chan = d.dg_raw || d.part_A || d.part_dt;
  float dA_acc = 0.f, ddt0 = 0.f, ddt1 = 0.f;
  if (n > 0 && need_chan) {
    const float negA = -expf(g.A_log[h]);
    const float2 bias = ld2(g.dt_bias + (size_t)h * K + k0);
    const GT* src = static_cast<const GT*>(g.g_raw) + row0 * K + k0;
    const float* dps = d.dg_pre ? d.dg_pre + row0 * K + k0 : nullptr;
    GT* dgr_out = d.dg_raw ? static_cast<GT*>(d.dg_raw) + row0 * K + k0 : nullptr;
    float acc0 = 0.f, acc1 = 0.f;  // reverse prefix of dg_pre
#pragma unroll 1
    for (int j0 = C - N; j0 >= 0; j0 -= N) {
      float2 x[N], dp[N];
      float dav[N];
      {
        const size_t off = (size_t)j0 * rs;
        const GT* px = src + off;
        const float* pd = dps ? dps + off : nullptr;
        const float* pa = d.da ? d.da + row0 + (size_t)j0 * g.H : nullptr;
#pragma unroll
        for (int j = 0; j < N; ++j, px += rs) {
          const bool in = j0 + j < n;
          x[j] = in ? ld2(px) : make_float2(0.f, 0.f);
          dp[j] = (in && pd) ? ld2(pd + (size_t)j * rs) : make_float2(0.f, 0.f);
          dav[j] = (in && pa) ? pa[(size_t)j * g.H] * (2.f / (float)K) : 0.f;
        }
      }
      GT* po = dgr_out ? dgr_out + (size_t)(j0 + N - 1) * rs : nullptr;
#pragma unroll
      for (int j = N - 1; j >= 0; --j, po -= rs) {
        if (j0 + j < n) {
          // e = e^x, u = 1 + e: softplus(x) = ln u, sigmoid(x) = e / u
          const float xb0 = x[j].x + bias.x, xb1 = x[j].y + bias.y;
          const float e0 = ex2a(xb0 * kLog2e), e1 = ex2a(xb1 * kLog2e);
          const float u0 = 1.f + e0, u1 = 1.f + e1;
          const float g0 = xb0 > 20.f ? negA * xb0 : (negA * kLn2) * __log2f(u0);
          const float g1 = xb1 > 20.f ? negA * xb1 : (negA * kLn2) * __log2f(u1);
          const float s0 = xb0 > 20.f ? 1.f : __fdividef(e0, u0);
          const float s1 = xb1 > 20.f ? 1.f : __fdividef(e1, u1);
          acc0 += dp[j].x;
          acc1 += dp[j].y;
          const float dg0 = fmaf(dav[j], ex2a(2.f * kLog2e * g0), acc0);
          const float dg1 = fmaf(dav[j], ex2a(2.f * kLog2e * g1), acc1);
          const float r0 = dg0 * negA * s0, r1 = dg1 * negA * s1;
          if (po) st_pair(po, r0, r1);
          dA_acc = fmaf(dg0, g0, fmaf(dg1, g1, dA_acc));
          ddt0 += r0;
          ddt1 += r1;
        }
      }
    }
  }
  const size_t np_row = (size_t)bc * g.H + h;
  if (d.part_dt) st_pair(d.part_dt + np_row * K + k0, ddt0, ddt1);
  // omega / r terms, one token per thread
  float swr = 0.f, srr = 0.f;
  for (int t = tid; t < n; t += NTH) {
    const size_t o = (size_t)b * g.stride_b + (size_t)(t0 + t) * g.stride_t + h;
    const size_t row = row0 + (size_t)t * g.H;
    float dwr = 0.f, drr = 0.f;
    if (d.domega) dwr = d.domega[row] * sigmoid_(ld_any(g.omega_r_raw, o, g.wr_bf16) + g.omega_bias[h]);
    if (d.dr) drr = d.dr[row] * sigmoid_(ld_any(g.omega_r_raw, o + g.H, g.wr_bf16) + g.r_bias[h]);
    if (d.domega_r_raw) {
      const size_t od = ((size_t)b * g.T + t0 + t) * (2 * (size_t)g.H) + h;
      st_any(d.domega_r_raw, od, g.wr_bf16, dwr);
      st_any(d.domega_r_raw, od + g.H, g.wr_bf16, drr);
    }
    swr += dwr;
    srr += drr;
  }
  if (d.part_A || d.part_wr) {
    // block sums of dA, domega_raw, dr_raw
    const float v0 = warp_sum(dA_acc), v1 = warp_sum(swr), v2 = warp_sum(srr);
    if (lane == 0) {
      red[warp * 3 + 0] = v0;
      red[warp * 3 + 1] = v1;
      red[warp * 3 + 2] = v2;
    }
    __syncthreads();
    if (tid == 0) {
      float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        s0 += red[w * 3 + 0];
        s1 += red[w * 3 + 1];
        s2 += red[w * 3 + 2];
      }
      if (d.part_A) d.part_A[np_row] = s0;
      if (d.part_wr) {
        d.part_wr[(size_t)bc * 2 * g.H + h] = s1;
        d.part_wr[(size_t)bc * 2 * g.H + g.H + h] = s2;
      }
    }
  }
  if (bc == 0 && tid == 0 && d.d_param) d.d_param[h] = d.d_init ? d.d_init[h] * sigmoid_(g.param[h]) : 0.f;
}

// out[i] = sum over the NP partial rows of part[row][i] (rows of `width`
// floats), for the requested outputs.  A CTA sums 32 consecutive outputs
// (lanes: consecutive addresses) with 8 row groups (warps) of NP / 8 rows
// each, then adds the 8 group sums in a fixed order.
constexpr int kRedCols = 32, kRedGroups = 8;
__device__ __forceinline__ void reduce_cols(const float* __restrict__ part, float* __restrict__ out, int width,
                                            int col, int NP, float (*sh)[kRedCols]) {
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  float s = 0.f;
  if (col < width)
#pragma unroll 4
    for (int p = ty; p < NP; p += kRedGroups) s += part[(size_t)p * width + col];
  sh[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && col < width) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kRedGroups; ++w) t += sh[w][tx];
    out[col] = t;
  }
}
// blockIdx.x: column blocks of ddt (H*K), then of dA (H), then of the two bias
// gradients (2H, one row of the omega / r partials)
__global__ void __launch_bounds__(kRedCols * kRedGroups) gate_reduce_kernel(
    const float* __restrict__ part_dt, float* __restrict__ ddt, int wdt, const float* __restrict__ part_A,
    float* __restrict__ dA, int wA, const float* __restrict__ part_wr, float* __restrict__ dwb,
    float* __restrict__ drb, int H, int NP) {
  __shared__ float sh[kRedGroups][kRedCols];
  const int nb_dt = (wdt + kRedCols - 1) / kRedCols, nb_A = (wA + kRedCols - 1) / kRedCols;
  const int blk = blockIdx.x, tx = threadIdx.x & 31;
  if (blk < nb_dt) {
    if (ddt) reduce_cols(part_dt, ddt, wdt, blk * kRedCols + tx, NP, sh);
  } else if (blk < nb_dt + nb_A) {
    if (dA) reduce_cols(part_A, dA, wA, (blk - nb_dt) * kRedCols + tx, NP, sh);
  } else if (dwb || drb) {
    // [NP][2H] partials: omega-bias columns first, then r-bias columns
    const int col = (blk - nb_dt - nb_A) * kRedCols + tx;
    const int ty = threadIdx.x >> 5;
    float s = 0.f;
    if (col < 2 * H)
#pragma unroll 4
      for (int p = ty; p < NP; p += kRedGroups) s += part_wr[(size_t)p * 2 * H + col];
    sh[ty][tx] = s;
    __syncthreads();
    if (ty == 0 && col < 2 * H) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kRedGroups; ++w) t += sh[w][tx];
      float* out = col < H ? dwb : drb;
      if (out) out[col < H ? col : col - H] = t;
    }
  }
}

// ---------------------------------------------------------------------------
// Diagonal frontend: _diag_kdn_frontend_precumsum_paired
// (lit_gpt/kdn_ops/diag_kdn_chunk.py:2471; kernels 1867-2051), 32-token chunks:
//   x = retention_raw + dt_bias[h, k],  ell = -exp(A_log[h]) softplus(x),
//   alpha = exp(ell),  ell_mem = ln max(alpha, 1e-6) (NaN passes),
//   g_cumsum = log2(e) * (inclusive prefix of ell_mem over the chunk),
//   omega = softplus(omega_raw),  r = 0.01 + softplus(r_raw),
//   initial_precision = 0.1 + softplus(param)
// Backward: mc = reverse prefix of d_g_cumsum (natural-log coordinates) over
// the chunk; dell = [alpha >= 1e-6] mc + d_alpha alpha (= (mc / alpha +
// d_alpha) alpha); dretention_raw = dell (-exp(A_log)) sigmoid(x);
// dA_log = sum dell ell; ddt_bias = sum_{b,t} dretention_raw;
// domega_raw = d_omega sigmoid(omega_raw); dr_raw = d_r sigmoid(r_raw);
// d_param = d_initial_precision sigmoid(param).  alpha is recomputed from
// retention_raw, so the backward needs no saved output.
constexpr int kDiagGateChunk = 32;
constexpr float kAlphaFloor = 1e-6f;

struct DiagGateArgs {
  const bf16 *ret, *wraw, *rraw;
  const float *A_log, *dt_bias, *param;
  int T, H, NT;
};

// Forward: CTA = (b, 32-token chunk, h), K / 2 threads with two channels
// each; 8 tokens of retention_raw and omega_raw are loaded per pass.
template <int K>
__global__ void __launch_bounds__(K / 2, 2048 / K) diag_gate_fwd_kernel(DiagGateArgs g, float* __restrict__ g_cumsum,
                                                                        float* __restrict__ alpha,
                                                                        float* __restrict__ omega,
                                                                        float* __restrict__ r,
                                                                        float* __restrict__ init_prec) {
  constexpr int C = kDiagGateChunk, N = 8, NTH = K / 2;
  const int bc = blockIdx.x / g.H, h = blockIdx.x - bc * g.H, tid = threadIdx.x, k0 = 2 * tid;
  const int b = g.NT ? bc / g.NT : 0, c = g.NT ? bc - b * g.NT : 0;
  const int t0 = c * C, n = min(C, g.T - t0);
  const size_t row0 = ((size_t)b * g.T + t0) * g.H + h;
  const size_t rs = (size_t)g.H * K;
  if (n > 0) {
    const float negA = -expf(g.A_log[h]);
    const float log_floor = logf(kAlphaFloor);
    const float2 bias = ld2(g.dt_bias + (size_t)h * K + k0);
    const size_t e0 = row0 * K + k0;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 1
    for (int j0 = 0; j0 < C; j0 += N) {
      float2 x[N], z[N];
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const bool in = j0 + j < n;
        const size_t e = e0 + (size_t)(j0 + j) * rs;
        x[j] = in ? ld2(g.ret + e) : make_float2(0.f, 0.f);
        z[j] = in ? ld2(g.wraw + e) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < N; ++j) {
        if (j0 + j < n) {
          const size_t e = e0 + (size_t)(j0 + j) * rs;
          const float l0 = gate_of(x[j].x + bias.x, negA), l1 = gate_of(x[j].y + bias.y, negA);
          const float a0 = ex2a(l0 * kLog2e), a1 = ex2a(l1 * kLog2e);
          s0 += a0 < kAlphaFloor ? log_floor : l0;  // a NaN alpha keeps its NaN ell
          s1 += a1 < kAlphaFloor ? log_floor : l1;
          st_pair(g_cumsum + e, s0 * kLog2e, s1 * kLog2e);
          st_pair(alpha + e, a0, a1);
          st_pair(omega + e, softplus_fla(z[j].x), softplus_fla(z[j].y));
        }
      }
    }
    for (int t = tid; t < n; t += NTH)
      r[row0 + (size_t)t * g.H] = 0.01f + softplus_fla(__bfloat162float(g.rraw[row0 + (size_t)t * g.H]));
  }
  if (bc == 0 && tid == 0) init_prec[h] = 0.1f + softplus_fla(g.param[h]);
}

struct DiagGateGrads {
  const float *d_gc, *d_alpha, *d_omega, *d_r, *d_init;  // nullable cotangents (contiguous)
  bf16 *dret, *domega_raw, *dr_raw;                      // nullable outputs, bf16 like the inputs
  float *part_A, *part_dt, *d_param;                     // nullable
};

// Backward: same CTA map as the forward; the chunk is walked from its last
// token down in passes of 8 tokens carrying the reverse prefix of d_g_cumsum.
// dA_log / ddt_bias leave per-CTA partial sums, summed by gate_reduce_kernel.
template <int K>
__global__ void __launch_bounds__(K / 2, 2048 / K) diag_gate_bwd_kernel(DiagGateArgs g, DiagGateGrads d) {
  constexpr int C = kDiagGateChunk, N = 8, NTH = K / 2, NW = NTH / 32;
  __shared__ float red[NW];
  const int bc = blockIdx.x / g.H, h = blockIdx.x - bc * g.H, tid = threadIdx.x, k0 = 2 * tid;
  const int warp = tid >> 5, lane = tid & 31;
  const int b = g.NT ? bc / g.NT : 0, c = g.NT ? bc - b * g.NT : 0;
  const int t0 = c * C, n = min(C, g.T - t0);
  const size_t row0 = ((size_t)b * g.T + t0) * g.H + h;
  const size_t rs = (size_t)g.H * K;
  const size_t e0 = row0 * K + k0;
  float dA_acc = 0.f, ddt0 = 0.f, ddt1 = 0.f;
  if (n > 0 && (d.d_gc || d.d_alpha) && (d.dret || d.part_A || d.part_dt)) {
    const float negA = -expf(g.A_log[h]);
    const float2 bias = ld2(g.dt_bias + (size_t)h * K + k0);
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 1
    for (int j0 = C - N; j0 >= 0; j0 -= N) {
      if (j0 >= n) continue;
      float2 x[N], dgc[N], da[N];
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const bool in = j0 + j < n;
        const size_t e = e0 + (size_t)(j0 + j) * rs;
        x[j] = in ? ld2(g.ret + e) : make_float2(0.f, 0.f);
        dgc[j] = (in && d.d_gc) ? ld2(d.d_gc + e) : make_float2(0.f, 0.f);
        da[j] = (in && d.d_alpha) ? ld2(d.d_alpha + e) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int j = N - 1; j >= 0; --j) {
        if (j0 + j < n) {
          // one e^x serves softplus (ln u) and sigmoid (e / u)
          const float xb0 = x[j].x + bias.x, xb1 = x[j].y + bias.y;
          const float ex0 = ex2a(xb0 * kLog2e), ex1 = ex2a(xb1 * kLog2e);
          const float u0 = 1.f + ex0, u1 = 1.f + ex1;
          const float l0 = xb0 > 20.f ? negA * xb0 : (negA * kLn2) * __log2f(u0);
          const float l1 = xb1 > 20.f ? negA * xb1 : (negA * kLn2) * __log2f(u1);
          const float sg0 = xb0 > 20.f ? 1.f : __fdividef(ex0, u0);
          const float sg1 = xb1 > 20.f ? 1.f : __fdividef(ex1, u1);
          const float a0 = ex2a(l0 * kLog2e), a1 = ex2a(l1 * kLog2e);
          acc0 += dgc[j].x;
          acc1 += dgc[j].y;
          const float dl0 = fmaf(da[j].x, a0, a0 >= kAlphaFloor ? acc0 : 0.f);
          const float dl1 = fmaf(da[j].y, a1, a1 >= kAlphaFloor ? acc1 : 0.f);
          const float r0 = dl0 * negA * sg0, r1 = dl1 * negA * sg1;
          if (d.dret) st_pair(d.dret + e0 + (size_t)(j0 + j) * rs, r0, r1);
          dA_acc = fmaf(dl0, l0, fmaf(dl1, l1, dA_acc));
          ddt0 += r0;
          ddt1 += r1;
        }
      }
    }
  }
  const size_t np_row = (size_t)bc * g.H + h;
  if (d.part_dt) st_pair(d.part_dt + np_row * K + k0, ddt0, ddt1);
  if (d.part_A) {
    const float v = warp_sum(dA_acc);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (tid == 0) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) s += red[w];
      d.part_A[np_row] = s;
    }
  }
  if (d.domega_raw && n > 0) {
#pragma unroll 1
    for (int j0 = 0; j0 < n; j0 += N) {
      float2 z[N], dw[N];
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const bool in = j0 + j < n;
        const size_t e = e0 + (size_t)(j0 + j) * rs;
        z[j] = in ? ld2(g.wraw + e) : make_float2(0.f, 0.f);
        dw[j] = in ? ld2(d.d_omega + e) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < N; ++j)
        if (j0 + j < n)
          st_pair(d.domega_raw + e0 + (size_t)(j0 + j) * rs, dw[j].x * sigmoid_(z[j].x), dw[j].y * sigmoid_(z[j].y));
    }
  }
  if (d.dr_raw)
    for (int t = tid; t < n; t += NTH) {
      const size_t row = row0 + (size_t)t * g.H;
      d.dr_raw[row] = __float2bfloat16_rn(d.d_r[row] * sigmoid_(__bfloat162float(g.rraw[row])));
    }
  if (bc == 0 && tid == 0 && d.d_param) d.d_param[h] = d.d_init[h] * sigmoid_(g.param[h]);
}

int gate_check(const char* what, int64_t B, int64_t T, int64_t H, int64_t K, const void* wr, int64_t sb, int64_t st) {
  if (B < 0 || T < 0 || H <= 0 || (K != 64 && K != 128))
    return set_error(KDN_ERR_INVALID, "%s: need B, T >= 0, H > 0 and K in {64, 128}", what);
  if (T > INT32_MAX || H * B * ((T + kGateChunk - 1) / kGateChunk) > INT32_MAX)
    return set_error(KDN_ERR_INVALID, "%s: size too large", what);
  if (B * T > 0 && (!wr || sb < 0 || st < 2 * H)) return set_error(KDN_ERR_INVALID, "%s: bad omega_r_raw strides", what);
  return KDN_OK;
}

}  // namespace
}  // namespace kdn

using namespace kdn;

extern "C" {

size_t kdn_iso_gate_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K) {
  if (B <= 0 || T <= 0 || H <= 0 || K <= 0) return 0;
  const int64_t NP = B * ((T + kGateChunk - 1) / kGateChunk);
  return align_up(sizeof(float) * (size_t)(NP * H * (K + 3)), 256);
}

int kdn_iso_gate_fwd(const void* g_raw, int g_raw_bf16, const void* omega_r_raw, int omega_r_raw_bf16,
                     int64_t omega_r_stride_b, int64_t omega_r_stride_t, const float* omega_bias,
                     const float* r_bias, const float* A_log, const float* dt_bias,
                     const float* initial_precision_param, float* g_cumsum, float* a, float* omega, float* r,
                     float* initial_precision, int64_t B, int64_t T, int64_t H, int64_t K, float omega_min,
                     float r_min, kdn_stream_t stream) {
  const char* what = "kdn_iso_gate_fwd";
  if (int rc = gate_check(what, B, T, H, K, omega_r_raw, omega_r_stride_b, omega_r_stride_t)) return rc;
  if (!omega_bias || !r_bias || !A_log || !dt_bias || !initial_precision_param || !initial_precision ||
      (B * T > 0 && (!g_raw || !g_cumsum || !a || !omega || !r)))
    return set_error(KDN_ERR_INVALID, "%s: null pointer", what);
  const int NT = (int)((T + kGateChunk - 1) / kGateChunk);
  GateArgs g{g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param,
             (long long)omega_r_stride_b, (long long)omega_r_stride_t, (int)T, (int)H, NT,
             g_raw_bf16 != 0, omega_r_raw_bf16 != 0};
  const unsigned grid = (unsigned)(H * (B * T > 0 ? B * NT : 1));
  cudaStream_t st = (cudaStream_t)stream;
  if (B * T == 0) g.NT = 0, g.T = 0;
  if (K == 128 && g.g_bf16)
    iso_gate_fwd_kernel<128, bf16><<<grid, 64, 0, st>>>(g, omega_min, r_min, g_cumsum, a, omega, r, initial_precision);
  else if (K == 128)
    iso_gate_fwd_kernel<128, float><<<grid, 64, 0, st>>>(g, omega_min, r_min, g_cumsum, a, omega, r, initial_precision);
  else if (g.g_bf16)
    iso_gate_fwd_kernel<64, bf16><<<grid, 32, 0, st>>>(g, omega_min, r_min, g_cumsum, a, omega, r, initial_precision);
  else
    iso_gate_fwd_kernel<64, float><<<grid, 32, 0, st>>>(g, omega_min, r_min, g_cumsum, a, omega, r, initial_precision);
  return check_launch("iso_gate_fwd_kernel");
}

int kdn_iso_gate_bwd(const void* g_raw, int g_raw_bf16, const void* omega_r_raw, int omega_r_raw_bf16,
                     int64_t omega_r_stride_b, int64_t omega_r_stride_t, const float* omega_bias,
                     const float* r_bias, const float* A_log, const float* dt_bias,
                     const float* initial_precision_param, const float* dg_pre_reverse, const float* da,
                     const float* domega, const float* dr, const float* d_initial_precision, void* dg_raw,
                     void* domega_r_raw, float* domega_bias, float* dr_bias, float* dA_log, float* ddt_bias,
                     float* d_initial_precision_param, int64_t B, int64_t T, int64_t H, int64_t K, void* workspace,
                     size_t workspace_bytes, kdn_stream_t stream) {
  const char* what = "kdn_iso_gate_bwd";
  if (int rc = gate_check(what, B, T, H, K, omega_r_raw, omega_r_stride_b, omega_r_stride_t)) return rc;
  if (!omega_bias || !r_bias || !A_log || !dt_bias || !initial_precision_param || (B * T > 0 && !g_raw))
    return set_error(KDN_ERR_INVALID, "%s: null pointer", what);
  if (workspace_bytes < kdn_iso_gate_workspace_bytes(B, T, H, K) || (B * T > 0 && !workspace))
    return set_error(KDN_ERR_WORKSPACE, "%s: workspace too small (kdn_iso_gate_workspace_bytes)", what);
  const bool empty = B * T == 0;
  const int NT = empty ? 0 : (int)((T + kGateChunk - 1) / kGateChunk);
  const int NP = empty ? 0 : (int)(B * NT);
  GateArgs g{g_raw, omega_r_raw, omega_bias, r_bias, A_log, dt_bias, initial_precision_param,
             (long long)omega_r_stride_b, (long long)omega_r_stride_t, empty ? 0 : (int)T, (int)H, NT,
             g_raw_bf16 != 0, omega_r_raw_bf16 != 0};
  float* part_dt = empty ? nullptr : static_cast<float*>(workspace);
  float* part_A = empty ? nullptr : part_dt + (size_t)NP * H * K;
  float* part_wr = empty ? nullptr : part_A + (size_t)NP * H;
  const bool need_wr = domega_bias || dr_bias;
  GateGrads d{dg_pre_reverse, da, domega, dr, d_initial_precision, empty ? nullptr : dg_raw,
              empty ? nullptr : domega_r_raw, need_wr ? part_wr : nullptr, dA_log ? part_A : nullptr,
              ddt_bias ? part_dt : nullptr, d_initial_precision_param};
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)(H * (empty ? 1 : NP));
  if (K == 128 && g.g_bf16)
    iso_gate_bwd_kernel<128, bf16><<<grid, 64, 0, st>>>(g, d);
  else if (K == 128)
    iso_gate_bwd_kernel<128, float><<<grid, 64, 0, st>>>(g, d);
  else if (g.g_bf16)
    iso_gate_bwd_kernel<64, bf16><<<grid, 32, 0, st>>>(g, d);
  else
    iso_gate_bwd_kernel<64, float><<<grid, 32, 0, st>>>(g, d);
  if (int rc = check_launch("iso_gate_bwd_kernel")) return rc;
  if (ddt_bias || dA_log || need_wr) {
    const int wdt = (int)(H * K), wA = (int)H;
    const int blocks = (wdt + kRedCols - 1) / kRedCols + (wA + kRedCols - 1) / kRedCols + (2 * (int)H + kRedCols - 1) / kRedCols;
    gate_reduce_kernel<<<blocks, kRedCols * kRedGroups, 0, st>>>(part_dt, ddt_bias, wdt, part_A, dA_log, wA, part_wr,
                                                                 domega_bias, dr_bias, (int)H, NP);
    return check_launch("gate_reduce_kernel");
  }
  return KDN_OK;
}

size_t kdn_diag_gate_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K) {
  if (B <= 0 || T <= 0 || H <= 0 || K <= 0) return 0;
  const int64_t NP = B * ((T + kDiagGateChunk - 1) / kDiagGateChunk);
  return align_up(sizeof(float) * (size_t)(NP * H * (K + 1)), 256);
}

static int diag_gate_check(const char* what, int64_t B, int64_t T, int64_t H, int64_t K) {
  if (B < 0 || T < 0 || H <= 0 || (K != 64 && K != 128))
    return set_error(KDN_ERR_INVALID, "%s: need B, T >= 0, H > 0 and K in {64, 128}", what);
  if (T > INT32_MAX || H * B * ((T + kDiagGateChunk - 1) / kDiagGateChunk) > INT32_MAX)
    return set_error(KDN_ERR_INVALID, "%s: size too large", what);
  return KDN_OK;
}

int kdn_diag_gate_fwd(const void* retention_raw, const void* omega_raw, const void* r_raw, const float* A_log,
                      const float* dt_bias, const float* initial_precision_param, float* g_cumsum, float* alpha,
                      float* omega, float* r, float* initial_precision, int64_t B, int64_t T, int64_t H, int64_t K,
                      kdn_stream_t stream) {
  const char* what = "kdn_diag_gate_fwd";
  if (int rc = diag_gate_check(what, B, T, H, K)) return rc;
  const bool empty = B * T == 0;
  if (!A_log || !dt_bias || !initial_precision_param || !initial_precision ||
      (!empty && (!retention_raw || !omega_raw || !r_raw || !g_cumsum || !alpha || !omega || !r)))
    return set_error(KDN_ERR_INVALID, "%s: null pointer", what);
  const int NT = empty ? 0 : (int)((T + kDiagGateChunk - 1) / kDiagGateChunk);
  DiagGateArgs g{static_cast<const bf16*>(retention_raw), static_cast<const bf16*>(omega_raw),
                 static_cast<const bf16*>(r_raw), A_log, dt_bias, initial_precision_param, empty ? 0 : (int)T,
                 (int)H, NT};
  const unsigned grid = (unsigned)(H * (empty ? 1 : B * NT));
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 128)
    diag_gate_fwd_kernel<128><<<grid, 64, 0, st>>>(g, g_cumsum, alpha, omega, r, initial_precision);
  else
    diag_gate_fwd_kernel<64><<<grid, 32, 0, st>>>(g, g_cumsum, alpha, omega, r, initial_precision);
  return check_launch("diag_gate_fwd_kernel");
}

int kdn_diag_gate_bwd(const void* retention_raw, const void* omega_raw, const void* r_raw, const float* A_log,
                      const float* dt_bias, const float* initial_precision_param, const float* d_g_cumsum,
                      const float* d_alpha, const float* d_omega, const float* d_r, const float* d_initial_precision,
                      void* dretention_raw, void* domega_raw, void* dr_raw, float* dA_log, float* ddt_bias,
                      float* d_initial_precision_param, int64_t B, int64_t T, int64_t H, int64_t K, void* workspace,
                      size_t workspace_bytes, kdn_stream_t stream) {
  const char* what = "kdn_diag_gate_bwd";
  if (int rc = diag_gate_check(what, B, T, H, K)) return rc;
  const bool empty = B * T == 0;
  if (!A_log || !dt_bias || !initial_precision_param ||
      (!empty && (!retention_raw || !omega_raw || !r_raw)) || (domega_raw && !d_omega) || (dr_raw && !d_r) ||
      (d_initial_precision_param && !d_initial_precision))
    return set_error(KDN_ERR_INVALID, "%s: null pointer (an output gradient needs its cotangent)", what);
  if (workspace_bytes < kdn_diag_gate_workspace_bytes(B, T, H, K) || (!empty && !workspace))
    return set_error(KDN_ERR_WORKSPACE, "%s: workspace too small (kdn_diag_gate_workspace_bytes)", what);
  const int NT = empty ? 0 : (int)((T + kDiagGateChunk - 1) / kDiagGateChunk);
  const int NP = (int)B * NT;
  DiagGateArgs g{static_cast<const bf16*>(retention_raw), static_cast<const bf16*>(omega_raw),
                 static_cast<const bf16*>(r_raw), A_log, dt_bias, initial_precision_param, empty ? 0 : (int)T,
                 (int)H, NT};
  float* part_dt = empty ? nullptr : static_cast<float*>(workspace);
  float* part_A = empty ? nullptr : part_dt + (size_t)NP * H * K;
  // without a decay cotangent dretention_raw is zero and dA_log / ddt_bias sum zeros
  DiagGateGrads d{d_g_cumsum, d_alpha, d_omega, d_r, d_initial_precision,
                  empty ? nullptr : static_cast<bf16*>(dretention_raw),
                  empty ? nullptr : static_cast<bf16*>(domega_raw), empty ? nullptr : static_cast<bf16*>(dr_raw),
                  dA_log ? part_A : nullptr, ddt_bias ? part_dt : nullptr, d_initial_precision_param};
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)(H * (empty ? 1 : NP));
  if (K == 128)
    diag_gate_bwd_kernel<128><<<grid, 64, 0, st>>>(g, d);
  else
    diag_gate_bwd_kernel<64><<<grid, 32, 0, st>>>(g, d);
  if (int rc = check_launch("diag_gate_bwd_kernel")) return rc;
  if (ddt_bias || dA_log) {  // with NP = 0 (empty input) the sums are zero
    const int wdt = (int)(H * K), wA = (int)H;
    const int blocks = (wdt + kRedCols - 1) / kRedCols + (wA + kRedCols - 1) / kRedCols;
    gate_reduce_kernel<<<blocks, kRedCols * kRedGroups, 0, st>>>(part_dt, ddt_bias, wdt, part_A, dA_log, wA, nullptr,
                                                                 nullptr, nullptr, (int)H, NP);
    return check_launch("gate_reduce_kernel");
  }
  return KDN_OK;
}

}  // extern "C"
