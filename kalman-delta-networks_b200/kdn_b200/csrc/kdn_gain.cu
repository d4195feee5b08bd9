// Covariance ("gain") scans of the isotropic and diagonal Kalman Delta Network.
//
// Both recurrences are Moebius maps of the covariance p, so a stream of T
// tokens is scanned in three phases: per-segment map composition, a carry over
// segments, then an exact per-token re-run from the carried covariance.  The
// backward is the reverse affine adjoint scan lambda_{t-1} = A_t lambda_t + B_t
// in the same three phases.
//
// Isotropic (one CTA per (b,h), one segment per thread, block-level scan of
// the 2x2 maps): lit_gpt/kdn_ops/iso_kdn_chunk.py:1464-1598 (forward) and
// 1667-1850 (backward) define the recurrence and its adjoint.
// Diagonal (one thread per key channel, 64-token segments, per-token channel
// reductions by warp transpose-reduce): diag_kdn_chunk.py:374-701 and the
// oracle diag_kdn_naive.py:256-276.
#include <mutex>

#include "kdn_common.cuh"

namespace kdn {
namespace {

constexpr int kDiagSeg = 64;

struct Mob {  // 2x2 Moebius map p -> (A p + B) / (C p + D)
  float A, B, C, D;
};

__device__ __forceinline__ Mob mob_mul(const Mob& x, const Mob& y) {  // x after y
  Mob z{x.A * y.A + x.B * y.C, x.A * y.B + x.B * y.D, x.C * y.A + x.D * y.C, x.C * y.B + x.D * y.D};
  float m = fmaxf(fmaxf(fabsf(z.A), fabsf(z.B)), fmaxf(fabsf(z.C), fabsf(z.D)));
  float inv = __fdividef(1.f, fmaxf(m, 1e-30f));
  return Mob{z.A * inv, z.B * inv, z.C * inv, z.D * inv};
}
__device__ __forceinline__ float mob_apply(const Mob& m, float p) { return (m.A * p + m.B) / (m.C * p + m.D); }

struct Aff {  // lambda -> A lambda + B
  float A, B;
};
__device__ __forceinline__ Aff aff_after(const Aff& f, const Aff& g) {  // f o g
  return Aff{f.A * g.A, f.A * g.B + f.B};
}

// ---------------------------------------------------------------------------
// Isotropic gain
// ---------------------------------------------------------------------------
// The rows [B,T,H] are contiguous over heads, so a warp takes one head per
// lane and reads one token of all its heads as one contiguous run (a thread
// per (b,h) reading its own tokens would touch one 32-byte sector per token
// and value, and the load unit, not memory, would bound it).  Each warp owns
// a segment of kIsoSeg tokens, kIsoWarps segments per CTA; the grid is
// (token blocks, B, head groups of 32).  Two launches per direction:
//   maps:  each segment's composed map and each CTA's total, to the workspace;
//   apply: the composition of every map before the segment (after it, in the
//          backward), then the exact per-token recurrence from that carry.
// The token blocks before a CTA are composed by its warps in kIsoWarps slices.
constexpr int kIsoSeg = 16, kIsoWarps = 8, kIsoBlockTok = kIsoSeg * kIsoWarps;

// Forward map of one token: p -> r z / (r + s z), z = a p + omega.
__device__ __forceinline__ Mob iso_tok_map(float a, float w, float r, float s) {
  return Mob{r * a, r * w, s * a, r + s * w};
}
// Adjoint of one token: lambda_{t-1} = A lambda_t + B (p_prev = p_{t-1}).
__device__ __forceinline__ Aff iso_tok_adj(float a, float w, float r, float db, float pp, float s) {
  const float z = a * pp + w;
  const float gi = 1.f / (r + z);
  const float pr = r / (r + s * z);
  return Aff{a * pr * pr, a * db * r * gi * gi};
}
__device__ __forceinline__ Mob as_mob(const float4& x) { return Mob{x.x, x.y, x.z, x.w}; }
__device__ __forceinline__ Aff as_aff(const float4& x) { return Aff{x.x, x.y}; }

// Workspace layout: [B][nblk][kIsoWarps][H] segment maps, then [B][nblk][H]
// CTA totals (float4: Moebius (A, B, C, D) or affine (A, B, -, -)).
struct IsoWs {
  float4* seg;
  float4* tot;
};
__host__ __device__ inline IsoWs iso_ws(void* ws, int B, int nblk, int H) {
  float4* seg = static_cast<float4*>(ws);
  return IsoWs{seg, seg + (size_t)B * nblk * kIsoWarps * H};
}

__global__ void __launch_bounds__(32 * kIsoWarps) iso_gain_fwd_maps_kernel(
    const float* __restrict__ a, const float* __restrict__ omega, const float* __restrict__ r, IsoWs ws, int T,
    int H, float s, const int* __restrict__ tok) {
  __shared__ Mob sm[kIsoWarps][32];
  const int blk = blockIdx.x, b = blockIdx.y, nblk = gridDim.x;
  // stream b: tokens [base, base + Tb) of the rows (a packed batch's sequence b)
  const int Tb = tok ? tok[b + 1] - tok[b] : T;
  const size_t base = tok ? (size_t)tok[b] : (size_t)b * T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = 32 * blockIdx.z + lane;
  const int ts = blk * kIsoBlockTok + warp * kIsoSeg;
  Mob m{1.f, 0.f, 0.f, 1.f};
  if (h < H) {
    float av[kIsoSeg], wv[kIsoSeg], rv[kIsoSeg];
#pragma unroll
    for (int j = 0; j < kIsoSeg; ++j) {
      const bool in = ts + j < Tb;
      const size_t off = (base + ts + j) * H + h;
      av[j] = in ? a[off] : 0.f;
      wv[j] = in ? omega[off] : 0.f;
      rv[j] = in ? r[off] : 1.f;
    }
#pragma unroll
    for (int j = 0; j < kIsoSeg; ++j)
      if (ts + j < Tb) m = mob_mul(iso_tok_map(av[j], wv[j], rv[j], s), m);
  }
  sm[warp][lane] = m;
  const size_t row = (size_t)b * nblk + blk;
  if (h < H) ws.seg[(row * kIsoWarps + warp) * H + h] = make_float4(m.A, m.B, m.C, m.D);
  __syncthreads();
  if (warp == 0 && h < H) {
    Mob t{1.f, 0.f, 0.f, 1.f};
#pragma unroll
    for (int w = 0; w < kIsoWarps; ++w) t = mob_mul(sm[w][lane], t);
    ws.tot[row * H + h] = make_float4(t.A, t.B, t.C, t.D);
  }
}

// T = 0 runs with one token block and no maps: only p_final is written.
__global__ void __launch_bounds__(32 * kIsoWarps) iso_gain_fwd_apply_kernel(
    const float* __restrict__ a, const float* __restrict__ omega, const float* __restrict__ r,
    const float* __restrict__ init_prec, const float* __restrict__ init_cov, IsoWs ws, float* __restrict__ gain,
    float* __restrict__ p_prev, float* __restrict__ p_final, int T, int H, float s, const int* __restrict__ tok) {
  __shared__ Mob part[kIsoWarps][32];
  const int blk = blockIdx.x, b = blockIdx.y, nblk = gridDim.x;
  // stream b: tokens [base, base + Tb) of the rows (a packed batch's sequence b)
  const int Tb = tok ? tok[b + 1] - tok[b] : T;
  const size_t base = tok ? (size_t)tok[b] : (size_t)b * T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = 32 * blockIdx.z + lane;
  const bool on = h < H;
  const int ts = blk * kIsoBlockTok + warp * kIsoSeg;
  // this segment's rows first: their latency overlaps the carry
  float av[kIsoSeg], wv[kIsoSeg], rv[kIsoSeg];
#pragma unroll
  for (int j = 0; j < kIsoSeg; ++j) {
    const bool in = on && ts + j < Tb;
    const size_t off = (base + ts + j) * H + h;
    av[j] = in ? a[off] : 0.f;
    wv[j] = in ? omega[off] : 0.f;
    rv[j] = in ? r[off] : 1.f;
  }
  // this warp's slice of the token blocks before this one
  Mob c{1.f, 0.f, 0.f, 1.f};
  if (on) {
    const int lo = (int)((int64_t)blk * warp / kIsoWarps), hi = (int)((int64_t)blk * (warp + 1) / kIsoWarps);
    for (int k = lo; k < hi; ++k) c = mob_mul(as_mob(ws.tot[((size_t)b * nblk + k) * H + h]), c);
  }
  part[warp][lane] = c;
  __syncthreads();
  const bool first = blk == 0 && warp == 0;
  if (!on || (ts >= Tb && !first)) return;
  Mob pre{1.f, 0.f, 0.f, 1.f};
#pragma unroll
  for (int w = 0; w < kIsoWarps; ++w) pre = mob_mul(part[w][lane], pre);
  const size_t row = (size_t)b * nblk + blk;
  for (int w = 0; w < warp; ++w) pre = mob_mul(as_mob(ws.seg[(row * kIsoWarps + w) * H + h]), pre);
  const float p0 = init_cov ? init_cov[(size_t)b * H + h] : 1.f / init_prec[h];
  float p = mob_apply(pre, p0);
#pragma unroll
  for (int j = 0; j < kIsoSeg; ++j) {
    if (ts + j < Tb) {
      const size_t off = (base + ts + j) * H + h;
      if (p_prev) p_prev[off] = p;
      const float z = av[j] * p + wv[j];
      const float beta = z / (rv[j] + z);
      gain[off] = beta;
      p = (s == 1.f) ? rv[j] * beta : rv[j] * z / (rv[j] + s * z);
    }
  }
  if (p_final && (Tb == 0 || (ts <= Tb - 1 && Tb - 1 < ts + kIsoSeg))) p_final[(size_t)b * H + h] = p;
}

__global__ void __launch_bounds__(32 * kIsoWarps) iso_gain_bwd_maps_kernel(
    const float* __restrict__ a, const float* __restrict__ omega, const float* __restrict__ r,
    const float* __restrict__ dgain, const float* __restrict__ p_prev, IsoWs ws, int T, int H, float s,
    const int* __restrict__ tok) {
  __shared__ Aff sm[kIsoWarps][32];
  const int blk = blockIdx.x, b = blockIdx.y, nblk = gridDim.x;
  // stream b: tokens [base, base + Tb) of the rows (a packed batch's sequence b)
  const int Tb = tok ? tok[b + 1] - tok[b] : T;
  const size_t base = tok ? (size_t)tok[b] : (size_t)b * T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = 32 * blockIdx.z + lane;
  const int ts = blk * kIsoBlockTok + warp * kIsoSeg;
  // lambda_{ts-1} = F_ts o ... o F_{te-1} (lambda_{te-1}): walking t downwards,
  // F_t goes on the outside
  Aff f{1.f, 0.f};
  if (h < H) {
    float av[kIsoSeg], wv[kIsoSeg], rv[kIsoSeg], dv[kIsoSeg], pv[kIsoSeg];
#pragma unroll
    for (int j = 0; j < kIsoSeg; ++j) {
      const bool in = ts + j < Tb;
      const size_t off = (base + ts + j) * H + h;
      av[j] = in ? a[off] : 0.f;
      wv[j] = in ? omega[off] : 0.f;
      rv[j] = in ? r[off] : 1.f;
      dv[j] = in ? dgain[off] : 0.f;
      pv[j] = in ? p_prev[off] : 0.f;
    }
#pragma unroll
    for (int j = kIsoSeg - 1; j >= 0; --j)
      if (ts + j < Tb) f = aff_after(iso_tok_adj(av[j], wv[j], rv[j], dv[j], pv[j], s), f);
  }
  sm[warp][lane] = f;
  const size_t row = (size_t)b * nblk + blk;
  if (h < H) ws.seg[(row * kIsoWarps + warp) * H + h] = make_float4(f.A, f.B, 0.f, 0.f);
  __syncthreads();
  if (warp == 0 && h < H) {
    Aff t{1.f, 0.f};
#pragma unroll
    for (int w = kIsoWarps - 1; w >= 0; --w) t = aff_after(sm[w][lane], t);
    ws.tot[row * H + h] = make_float4(t.A, t.B, 0.f, 0.f);
  }
}

// T = 0 runs with one token block and no maps: the cotangent of p_{-1} is
// d_final_cov itself.
__global__ void __launch_bounds__(32 * kIsoWarps) iso_gain_bwd_apply_kernel(
    const float* __restrict__ a, const float* __restrict__ omega, const float* __restrict__ r,
    const float* __restrict__ init_prec, const float* __restrict__ dgain, const float* __restrict__ p_prev,
    const float* __restrict__ d_final_cov, const bool has_init_cov, float* __restrict__ d_init_cov, IsoWs ws,
    float* __restrict__ da, float* __restrict__ domega, float* __restrict__ dr, float* __restrict__ dinit, int T,
    int H, float s, const int* __restrict__ tok) {
  __shared__ Aff part[kIsoWarps][32];
  const int blk = blockIdx.x, b = blockIdx.y, nblk = gridDim.x;
  // stream b: tokens [base, base + Tb) of the rows (a packed batch's sequence b)
  const int Tb = tok ? tok[b + 1] - tok[b] : T;
  const size_t base = tok ? (size_t)tok[b] : (size_t)b * T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = 32 * blockIdx.z + lane;
  const bool on = h < H;
  const int ts = blk * kIsoBlockTok + warp * kIsoSeg;
  float av[kIsoSeg], wv[kIsoSeg], rv[kIsoSeg], dv[kIsoSeg], pv[kIsoSeg];
#pragma unroll
  for (int j = 0; j < kIsoSeg; ++j) {
    const bool in = on && ts + j < Tb;
    const size_t off = (base + ts + j) * H + h;
    av[j] = in ? a[off] : 0.f;
    wv[j] = in ? omega[off] : 0.f;
    rv[j] = in ? r[off] : 1.f;
    dv[j] = in ? dgain[off] : 0.f;
    pv[j] = in ? p_prev[off] : 0.f;
  }
  // this warp's slice of the token blocks after this one, composed as
  // Tot_lo o ... o Tot_{hi-1}
  Aff c{1.f, 0.f};
  if (on) {
    const int n = nblk - 1 - blk;
    const int lo = blk + 1 + (int)((int64_t)n * warp / kIsoWarps);
    const int hi = blk + 1 + (int)((int64_t)n * (warp + 1) / kIsoWarps);
    for (int k = hi - 1; k >= lo; --k) c = aff_after(as_aff(ws.tot[((size_t)b * nblk + k) * H + h]), c);
  }
  part[warp][lane] = c;
  __syncthreads();
  const bool first = blk == 0 && warp == 0;
  if (!on || (ts >= Tb && !first)) return;
  Aff suf{1.f, 0.f};
#pragma unroll
  for (int w = kIsoWarps - 1; w >= 0; --w) suf = aff_after(part[w][lane], suf);
  if (Tb > 0) {
    const size_t row = (size_t)b * nblk + blk;
    for (int w = kIsoWarps - 1; w > warp; --w) suf = aff_after(as_aff(ws.seg[(row * kIsoWarps + w) * H + h]), suf);
  }
  // lambda after the segment's last token (d_final_cov: the cotangent of p_{T-1}, 0 without one)
  float lam = suf.A * (d_final_cov ? d_final_cov[(size_t)b * H + h] : 0.f) + suf.B;
#pragma unroll
  for (int j = kIsoSeg - 1; j >= 0; --j) {
    if (ts + j < Tb) {
      const size_t off = (base + ts + j) * H + h;
      const float at = av[j], wt = wv[j], rt = rv[j], dbt = dv[j], pp = pv[j];
      const float z = at * pp + wt;
      float zbar, drt;
      if (s == 1.f) {
        const float inv = 1.f / (rt + z), inv2 = inv * inv;
        zbar = (dbt + rt * lam) * rt * inv2;
        drt = z * (lam * z - dbt) * inv2;
      } else {
        const float gi = 1.f / (rt + z), gi2 = gi * gi;
        const float pi = 1.f / (rt + s * z), pi2 = pi * pi;
        zbar = dbt * rt * gi2 + lam * rt * rt * pi2;
        drt = -dbt * z * gi2 + lam * s * z * z * pi2;
      }
      da[off] = zbar * pp;
      domega[off] = zbar;
      dr[off] = drt;
      lam = at * zbar;
    }
  }
  if (first) {
    if (d_init_cov) d_init_cov[(size_t)b * H + h] = lam;  // d L / d p_{-1}
    if (!has_init_cov) {
      const float ip = init_prec[h];
      atomicAdd(dinit + h, -lam / (ip * ip));
    }
  }
}

// The whole segment's map per (b, h) from the block totals of a maps launch
// (sequence parallelism): forward M_{n-1} o ... o M_0 as (A, B, C, D);
// backward (A, B) with lambda_in = A lambda_end + B, composed from the last
// block down, the order of the apply kernels.
__global__ void iso_gain_fwd_total_kernel(IsoWs ws, float4* __restrict__ total, int nblk, int B, int H) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * H) return;
  const int b = i / H, h = i - b * H;
  Mob m{1.f, 0.f, 0.f, 1.f};
  for (int k = 0; k < nblk; ++k) m = mob_mul(as_mob(ws.tot[((size_t)b * nblk + k) * H + h]), m);
  total[i] = make_float4(m.A, m.B, m.C, m.D);
}
__global__ void iso_gain_bwd_total_kernel(IsoWs ws, float2* __restrict__ total, int nblk, int B, int H) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * H) return;
  const int b = i / H, h = i - b * H;
  Aff f{1.f, 0.f};
  for (int k = nblk - 1; k >= 0; --k) f = aff_after(as_aff(ws.tot[((size_t)b * nblk + k) * H + h]), f);
  total[i] = make_float2(f.A, f.B);
}

// Host side: workspace size and launch grid.
size_t iso_ws_bytes(int64_t B, int64_t T, int64_t H) {
  if (B <= 0 || T <= 0 || H <= 0) return 0;
  const int64_t nblk = (T + kIsoBlockTok - 1) / kIsoBlockTok;
  return align_up(sizeof(float4) * (size_t)(B * nblk * (kIsoWarps + 1) * H), 256);
}

int iso_grid(const char* what, int64_t B, int64_t T, int64_t H, void* ws, size_t ws_bytes, dim3* grid) {
  if (T > INT32_MAX || B > 65535 || (H + 31) / 32 > 65535 || H > INT32_MAX)
    return set_error(KDN_ERR_INVALID, "%s: size too large", what);
  if (ws_bytes < iso_ws_bytes(B, T, H) || (T > 0 && !ws))
    return set_error(KDN_ERR_WORKSPACE, "%s: workspace too small (kdn_iso_gain_workspace_bytes)", what);
  *grid = dim3(T > 0 ? (unsigned)((T + kIsoBlockTok - 1) / kIsoBlockTok) : 1u, (unsigned)B, (unsigned)((H + 31) / 32));
  return KDN_OK;
}

// ---------------------------------------------------------------------------
// Diagonal gain
// ---------------------------------------------------------------------------
// The diagonal kernels' inputs for TT consecutive tokens of a segment, staged
// in shared memory by cp.async: NA per-channel fp32 rows (k, alpha, omega, and
// in the backward dkappa and p_prev), optionally the bf16 omega_raw rows (WR)
// and the per-token (D, G) (DG), and r.  NS - 1 tiles are in flight while a
// CTA runs the sequential chain of the current one, and none of them occupies
// registers.  Every stage is refilled only after the block barrier that ends
// the previous use of it.  V16: every row pointer is 16-byte aligned and a
// thread copies 16 bytes (four channels) at a time; otherwise each thread
// copies its own channel's 4 bytes (omega_raw is then read where it is used),
// which is slower (gain backward 0.61 against 0.34 ms at B=4, T=4096, H=18).
// Tile and stage counts by timing at that shape: backward 8 x 2 (0.334 ms;
// 4 x 3: 0.347, 4 x 2: 0.343, 2 x 3: 0.356; the register-tile kernels they
// replaced: 0.494), forward 8 x 2 (0.241 ms; 4 x 3: 0.244, 2 x 4: 0.247,
// 4 x 2: 0.248; register tiles: 0.269-0.302).
constexpr int kGainTile = 8, kGainStages = 2;   // backward kernels
constexpr int kGainTileF = 8, kGainStagesF = 2;  // forward kernels
// Segment maps a carry kernel loads ahead of the sequential chain that applies them.
constexpr int kCarryBatch = 16;
template <int K, int TT, int NA, bool WR, bool DG>
struct alignas(16) GainStage {
  float row[NA][TT][K];
  bf16 wr[WR ? TT : 1][K];
  float2 dg[TT];
  float r[TT];

  // rows [ts, ts + m) of the segment starting at row0 (row stride H); tok0
  // indexes (D, G) of the segment's first token
  template <bool V16>
  __device__ __forceinline__ void load(const float* const (&src)[NA], const bf16* __restrict__ omega_raw,
                                       const float* __restrict__ rr, const float2* __restrict__ dg_tok, size_t row0,
                                       int H, int ts, int m, size_t tok0) {
    const int c = threadIdx.x;
    if constexpr (V16) {
      constexpr int P = K / 4, NP = (TT * P + K - 1) / K;  // 16-byte pieces per fp32 row; per thread
#pragma unroll
      for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          const int e = c + i * K, j = e / P, pc = e - j * P;
          if (e < TT * P && j < m) cp_async16(&row[a][j][4 * pc], src[a] + (row0 + (size_t)(ts + j) * H) * K + 4 * pc);
        }
      if constexpr (WR) {
        constexpr int PW = K / 8, NW = (TT * PW + K - 1) / K;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
          const int e = c + i * K, j = e / PW, pc = e - j * PW;
          if (e < TT * PW && j < m) cp_async16(&wr[j][8 * pc], omega_raw + (row0 + (size_t)(ts + j) * H) * K + 8 * pc);
        }
      }
    } else {
#pragma unroll
      for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int j = 0; j < TT; ++j)
          if (j < m) cp_async4(&row[a][j][c], src[a] + (row0 + (size_t)(ts + j) * H) * K + c);
    }
    if (c < m) {
      cp_async4(&r[c], rr + row0 + (size_t)(ts + c) * H);
      if constexpr (DG) cp_async8(&dg[c], dg_tok + tok0 + ts + c);
    }
  }
};

// Tokens [t0, t0 + n) of 64-token segment `seg` (a global chunk of a packed
// batch when v is on) and the index of its (sequence, head) stream.
__device__ __forceinline__ void seg_span(const Varlen& v, int seg, int T, int H, int bh, int& t0, int& n, int& sh) {
  if (v.on()) {
    int s;
    varlen_span(v, seg, t0, n, s);
    sh = s * H + bh;  // B = 1: bh is the head
  } else {
    t0 = seg * kDiagSeg;
    n = min(kDiagSeg, T - t0);
    sh = bh;
  }
}

// Forward pass A: each segment's composed covariance map.
template <int K, bool V16>
__global__ void __launch_bounds__(K) diag_gain_map_kernel(const float* __restrict__ k, const float* __restrict__ alpha,
                                                          const float* __restrict__ omega, const float* __restrict__ r,
                                                          float4* __restrict__ maps, int T, int H, int nseg,
                                                          Varlen v) {
  constexpr int TT = kGainTileF, NS = kGainStagesF;
  using Stage = GainStage<K, TT, 3, false, false>;
  __shared__ Stage stg[NS];
  const int seg = blockIdx.x, bh = blockIdx.y, b = bh / H, h = bh - b * H, c = threadIdx.x;
  int t0, n, sh;
  seg_span(v, seg, T, H, bh, t0, n, sh);
  const size_t row0 = ((size_t)b * T + t0) * H + h;
  const float* const src[3] = {k, alpha, omega};
  const int ntiles = (n + TT - 1) / TT;
  auto issue = [&](int it) {
    if (it < ntiles) stg[it % NS].template load<V16>(src, nullptr, r, nullptr, row0, H, it * TT, min(TT, n - it * TT), 0);
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < NS - 1; ++i) issue(i);
  Mob m{1.f, 0.f, 0.f, 1.f};
  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait_group<NS - 2>();
    __syncthreads();
    issue(it + NS - 1);
    const Stage& S = stg[it % NS];
    const int ts = it * TT;
#pragma unroll
    for (int j = 0; j < TT; ++j) {
      if (ts + j < n) {
        const float kt = S.row[0][j][c], at = S.row[1][j][c], wt = S.row[2][j][c];
        const float a2 = at * at, u = __fdividef((float)K * kt * kt, S.r[j]);
        m = mob_mul(Mob{a2, wt, u * a2, 1.f + u * wt}, m);
      }
    }
  }
  cp_async_wait_all();
  maps[((size_t)bh * nseg + seg) * K + c] = make_float4(m.A, m.B, m.C, m.D);
}

template <int K>
__global__ void __launch_bounds__(K) diag_gain_carry_kernel(const float4* __restrict__ maps,
                                                            const float* __restrict__ init_prec,
                                                            const float* __restrict__ init_cov,
                                                            float* __restrict__ carry, float* __restrict__ p_final,
                                                            int H, int nseg, Varlen v) {
  // one (sequence, head) stream; its segments are [s0, s1) of the (b, h) row
  // of segment maps (packed batch: the head's row, the sequence's chunks)
  const int sh = blockIdx.x, h = sh % H, c = threadIdx.x;
  const int row = v.on() ? h : sh, s0 = v.on() ? v.chunk[sh / H] : 0, s1 = v.on() ? v.chunk[sh / H + 1] : nseg;
  float p = init_cov ? init_cov[(size_t)sh * K + c] : 1.f / init_prec[h];
  // the maps do not depend on p: kCarryBatch of them are loaded before they are applied
  for (int s = s0; s < s1; s += kCarryBatch) {
    float4 m[kCarryBatch];
#pragma unroll
    for (int i = 0; i < kCarryBatch; ++i)
      if (s + i < s1) m[i] = maps[((size_t)row * nseg + s + i) * K + c];
#pragma unroll
    for (int i = 0; i < kCarryBatch; ++i)
      if (s + i < s1) {
        carry[((size_t)row * nseg + s + i) * K + c] = p;
        p = mob_apply(Mob{m[i].x, m[i].y, m[i].z, m[i].w}, p);
      }
  }
  if (p_final) p_final[(size_t)sh * K + c] = p;
}

// Forward pass C: the exact per-token recurrence of every segment from its
// carried covariance; writes kappa and the covariance before every token.
template <int K, bool V16>
__global__ void __launch_bounds__(K) diag_gain_emit_kernel(const float* __restrict__ k, const float* __restrict__ alpha,
                                                           const float* __restrict__ omega,
                                                           const float* __restrict__ r,
                                                           const float* __restrict__ carry,
                                                           float* __restrict__ kappa, float* __restrict__ p_prev,
                                                           int T, int H, int nseg, Varlen v) {
  constexpr int TT = kGainTileF, NS = kGainStagesF;
  using Stage = GainStage<K, TT, 3, false, false>;
  __shared__ Stage stg[NS];
  __shared__ float red[K / 32 * TT];
  __shared__ float tok[TT];
  const int seg = blockIdx.x, bh = blockIdx.y, b = bh / H, h = bh - b * H, c = threadIdx.x;
  int t0, n, sh;
  seg_span(v, seg, T, H, bh, t0, n, sh);
  const size_t row0 = ((size_t)b * T + t0) * H + h;
  const float* const src[3] = {k, alpha, omega};
  const int ntiles = (n + TT - 1) / TT;
  auto issue = [&](int it) {
    if (it < ntiles) stg[it % NS].template load<V16>(src, nullptr, r, nullptr, row0, H, it * TT, min(TT, n - it * TT), 0);
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < NS - 1; ++i) issue(i);
  float p = carry[((size_t)bh * nseg + seg) * K + c];
  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait_group<NS - 2>();
    __syncthreads();
    issue(it + NS - 1);
    const Stage& S = stg[it % NS];
    const int ts = it * TT;
    float num[TT], pk2[TT];
#pragma unroll
    for (int j = 0; j < TT; ++j) {
      num[j] = 0.f;
      pk2[j] = 0.f;
      if (ts + j < n) {
        p_prev[(row0 + (size_t)(ts + j) * H) * K + c] = p;  // for the backward
        const float kt = S.row[0][j][c], at = S.row[1][j][c];
        const float ph = at * at * p + S.row[2][j][c];
        const float ksq = kt * kt;
        num[j] = ph * kt;
        pk2[j] = ph * ksq;
        const float u = __fdividef((float)K * ksq, S.r[j]);
        p = __fdividef(ph, 1.f + u * ph);
      }
    }
    block_token_sums<K, TT>(pk2, red, tok);
#pragma unroll
    for (int j = 0; j < TT; ++j)
      if (ts + j < n) kappa[(row0 + (size_t)(ts + j) * H) * K + c] = __fdividef(num[j], S.r[j] + tok[j]);
  }
  cp_async_wait_all();
}

// Backward pass A: per segment, form the per-token channel reductions
// D_t = r_t + sum p_hat k^2 and G_t = sum dkappa * kappa from the covariance
// before every token (p_prev, saved by the forward), and compose the reverse
// affine maps.  The tokens of a tile are independent; only the maps compose in
// order.
template <int K, bool V16>
__global__ void __launch_bounds__(K) diag_gain_bwd_map_kernel(
    const float* __restrict__ k, const float* __restrict__ alpha, const float* __restrict__ omega,
    const float* __restrict__ r, const float* __restrict__ dkappa, const float* __restrict__ p_prev,
    float2* __restrict__ maps, float2* __restrict__ dg_tok, int T, int H, int nseg, Varlen v) {
  constexpr int TT = kGainTile, NS = kGainStages;
  using Stage = GainStage<K, TT, 5, false, false>;
  __shared__ Stage stg[NS];
  __shared__ float red[K / 32 * 2 * TT];
  __shared__ float tok[2 * TT];  // [sum p_hat k^2 | sum dkappa p_hat k] per token
  const int seg = blockIdx.x, bh = blockIdx.y, b = bh / H, h = bh - b * H, c = threadIdx.x;
  int t0, n, sh;
  seg_span(v, seg, T, H, bh, t0, n, sh);
  const size_t row0 = ((size_t)b * T + t0) * H + h;
  const float Kf = (float)K;
  const float* const src[5] = {k, alpha, omega, dkappa, p_prev};
  const int ntiles = (n + TT - 1) / TT;
  // tile it into stage it % NS; every call commits one group (empty past the end)
  auto issue = [&](int it) {
    if (it < ntiles) stg[it % NS].template load<V16>(src, nullptr, r, nullptr, row0, H, it * TT, min(TT, n - it * TT), 0);
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < NS - 1; ++i) issue(i);
  Aff comp{1.f, 0.f};
  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait_group<NS - 2>();  // tile it has landed (this thread's copies) ...
    __syncthreads();                // ... everyone's, and no thread still reads tile it - 1
    issue(it + NS - 1);             // into the stage of tile it - 1
    const Stage& S = stg[it % NS];
    const int ts = it * TT;
    float x[2 * TT];
#pragma unroll
    for (int j = 0; j < TT; ++j) {
      x[j] = 0.f;
      x[TT + j] = 0.f;
      if (ts + j < n) {
        const float kt = S.row[0][j][c], at = S.row[1][j][c];
        const float ph = at * at * S.row[4][j][c] + S.row[2][j][c];
        x[j] = ph * kt * kt;
        x[TT + j] = S.row[3][j][c] * ph * kt;
      }
    }
    block_token_sums<K, 2 * TT>(x, red, tok);
#pragma unroll
    for (int j = 0; j < TT; ++j) {
      if (ts + j < n) {
        const float kt = S.row[0][j][c], rt = S.r[j];
        const float D = rt + tok[j], iD = __fdividef(1.f, D);
        const float G = tok[TT + j] * iD;
        if (c == 0) dg_tok[(size_t)bh * T + t0 + ts + j] = make_float2(D, G);
        const float a2 = S.row[1][j][c] * S.row[1][j][c];
        const float ph = a2 * S.row[4][j][c] + S.row[2][j][c];
        const float ihh = __fdividef(1.f, 1.f + __fdividef(Kf * kt * kt, rt) * ph);
        const float pbar_gain = (S.row[3][j][c] * kt - kt * kt * G) * iD;
        comp = aff_after(comp, Aff{a2 * ihh * ihh, a2 * pbar_gain});
      }
    }
  }
  cp_async_wait_all();  // only empty groups can be left
  maps[((size_t)bh * nseg + seg) * K + c] = make_float2(comp.A, comp.B);
}

template <int K>
__global__ void __launch_bounds__(K) diag_gain_bwd_carry_kernel(const float2* __restrict__ maps,
                                                                const float* __restrict__ d_final_cov,
                                                                float* __restrict__ lam_carry, int H, int nseg,
                                                                Varlen v) {
  const int sh = blockIdx.x, h = sh % H, c = threadIdx.x;
  const int row = v.on() ? h : sh, s0 = v.on() ? v.chunk[sh / H] : 0, s1 = v.on() ? v.chunk[sh / H + 1] : nseg;
  float lam = d_final_cov ? d_final_cov[(size_t)sh * K + c] : 0.f;
  for (int s = s1 - 1; s >= s0; s -= kCarryBatch) {
    float2 m[kCarryBatch];
#pragma unroll
    for (int i = 0; i < kCarryBatch; ++i)
      if (s - i >= s0) m[i] = maps[((size_t)row * nseg + s - i) * K + c];
#pragma unroll
    for (int i = 0; i < kCarryBatch; ++i)
      if (s - i >= s0) {
        lam_carry[((size_t)row * nseg + s - i) * K + c] = lam;
        lam = m[i].x * lam + m[i].y;
      }
  }
}

// Composed covariance map of a whole stream (sequence parallelism): the
// segment maps M_{n-1} o ... o M_0 per (b, h, channel), normalised like every
// composition here.
template <int K>
__global__ void __launch_bounds__(K) diag_gain_total_kernel(const float4* __restrict__ maps,
                                                            float4* __restrict__ total, int nseg) {
  const int bh = blockIdx.x, c = threadIdx.x;
  Mob m{1.f, 0.f, 0.f, 1.f};
  for (int s = 0; s < nseg; ++s) {
    const float4 x = maps[((size_t)bh * nseg + s) * K + c];
    m = mob_mul(Mob{x.x, x.y, x.z, x.w}, m);
  }
  total[(size_t)bh * K + c] = make_float4(m.A, m.B, m.C, m.D);
}

// Composed adjoint map of a whole stream: lambda_in = A lambda_out + B with
// (A, B) = m_0 o m_1 o ... o m_{n-1} of the segment maps.
template <int K>
__global__ void __launch_bounds__(K) diag_gain_bwd_total_kernel(const float2* __restrict__ maps,
                                                                float2* __restrict__ total, int nseg) {
  const int bh = blockIdx.x, c = threadIdx.x;
  Aff f{1.f, 0.f};
  for (int s = nseg - 1; s >= 0; --s) {
    const float2 m = maps[((size_t)bh * nseg + s) * K + c];
    f = aff_after(Aff{m.x, m.y}, f);
  }
  total[(size_t)bh * K + c] = make_float2(f.A, f.B);
}

__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// Backward pass B: the reverse adjoint per channel over tiles of TT tokens,
// last tile first, from the carried lambda of the segment, with the input
// gradients and the fused softplus VJPs.
template <int K, bool V16>
__global__ void __launch_bounds__(K) diag_gain_bwd_emit_kernel(
    const float* __restrict__ k, const float* __restrict__ alpha, const float* __restrict__ omega,
    const float* __restrict__ r, const float* __restrict__ init_prec, const bf16* __restrict__ omega_raw,
    const bf16* __restrict__ r_raw, const float* __restrict__ dkappa, const float* __restrict__ p_prev,
    const float* __restrict__ lam_carry, const float2* __restrict__ dg_tok, float* __restrict__ dk_out,
    float* __restrict__ dalpha, bf16* __restrict__ domega_raw, bf16* __restrict__ dr_raw,
    float* __restrict__ dinit, float* __restrict__ d_init_cov, int T, int H, int nseg, Varlen v) {
  constexpr int TT = kGainTile, NS = kGainStages;
  using Stage = GainStage<K, TT, 5, V16, true>;
  __shared__ Stage stg[NS];
  __shared__ float red[K / 32 * TT];
  __shared__ float tok[TT];
  const int seg = blockIdx.x, bh = blockIdx.y, b = bh / H, h = bh - b * H, c = threadIdx.x;
  int t0, n, sh;
  seg_span(v, seg, T, H, bh, t0, n, sh);
  const bool first = v.on() ? seg == v.chunk[sh / H] : seg == 0;  // the stream's first segment
  const size_t row0 = ((size_t)b * T + t0) * H + h, tok0 = (size_t)bh * T + t0;
  const float Kf = (float)K;
  const float* const src[5] = {k, alpha, omega, dkappa, p_prev};
  const int ntiles = (n + TT - 1) / TT, last = (ntiles - 1) * TT;
  // tile it (tokens from last - it * TT) into stage it % NS; one group per call
  auto issue = [&](int it) {
    if (it < ntiles) {
      const int ts = last - it * TT;
      stg[it % NS].template load<V16>(src, omega_raw, r, dg_tok, row0, H, ts, min(TT, n - ts), tok0);
    }
    cp_async_commit();
  };
  float lam = lam_carry[((size_t)bh * nseg + seg) * K + c];
#pragma unroll
  for (int i = 0; i < NS - 1; ++i) issue(i);
  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait_group<NS - 2>();
    __syncthreads();
    issue(it + NS - 1);
    const Stage& S = stg[it % NS];
    const int ts = last - it * TT;
    float ur[TT];
#pragma unroll
    for (int jj = TT - 1; jj >= 0; --jj) {
      ur[jj] = 0.f;
      if (ts + jj < n) {
        const size_t row = row0 + (size_t)(ts + jj) * H;
        const float kt = S.row[0][jj][c], at = S.row[1][jj][c], wt = S.row[2][jj][c], rt = S.r[jj];
        const float dk = S.row[3][jj][c], pp = S.row[4][jj][c];
        const float D = S.dg[jj].x, G = S.dg[jj].y, iD = __fdividef(1.f, D), ir = __fdividef(1.f, rt);
        float wr;
        if constexpr (V16) {
          wr = __bfloat162float(S.wr[jj][c]);
        } else {
          wr = __bfloat162float(omega_raw[row * K + c]);
        }
        const float a2 = at * at, ksq = kt * kt;
        const float ph = a2 * pp + wt;
        const float u = Kf * ksq * ir;
        const float ihh = __fdividef(1.f, 1.f + u * ph);
        const float pnext = ph * ihh;
        const float pbar_gain = (dk * kt - ksq * G) * iD;
        const float kbar_gain = (dk * ph - 2.f * ph * kt * G) * iD;
        const float pbar_tot = pbar_gain + lam * ihh * ihh;
        const float ubar = -lam * pnext * pnext;
        dk_out[row * K + c] = kbar_gain + ubar * (2.f * Kf * kt * ir);
        dalpha[row * K + c] = 2.f * at * pp * pbar_tot;
        domega_raw[row * K + c] = __float2bfloat16_rn(pbar_tot * sigmoidf_(wr));
        ur[jj] = -ubar * u * ir;
        lam = a2 * pbar_tot;
      }
    }
    block_token_sums<K, TT>(ur, red, tok);
    if (c < TT && ts + c < n) {
      const size_t row = row0 + (size_t)(ts + c) * H;
      const float2 DG = S.dg[c];
      const float drt = tok[c] - __fdividef(DG.y, DG.x);
      dr_raw[row] = __float2bfloat16_rn(drt * sigmoidf_(__bfloat162float(r_raw[row])));
    }
  }
  cp_async_wait_all();
  if (first && d_init_cov) d_init_cov[(size_t)sh * K + c] = lam;  // d L / d p_{-1}
  if (first && dinit) {
    // p_{-1} = 1/mu, so d mu = -sum_c lambda_{-1,c} p_{-1,c}^2
    const float p0 = p_prev[row0 * K + c];
    float x = -lam * p0 * p0;
    x = warp_sum(x);
    if ((c & 31) == 0) atomicAdd(dinit + h, x);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Scratch of kdn_diag_gain_fwd_noalloc: the per-segment covariance maps, in a
// file-scope device array instead of caller workspace.  Every GPU that loads
// the library holds these 16 MiB until the process exits.
// ---------------------------------------------------------------------------
constexpr int64_t kNoAllocMapEntries = 1 << 20;  // float4 entries = B*H*ceil(T/64)*K at most
static __device__ __align__(256) float4 g_noalloc_maps[kNoAllocMapEntries];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float4* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_maps on the current device.  In host code the
// array's name is only a host-side stand-in; the real address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
int noalloc_maps(float4** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(KDN_ERR_INVALID, "kdn_diag_gain_fwd_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&ptr, g_noalloc_maps);
    if (rc != cudaSuccess || !ptr)
      return set_error(KDN_ERR_CUDA, "kdn_diag_gain_fwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(rc));
    g_noalloc_ptr[dev] = static_cast<float4*>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return KDN_OK;
}
}  // namespace
}  // namespace kdn

using namespace kdn;

extern "C" {

size_t kdn_iso_gain_workspace_bytes(int64_t B, int64_t T, int64_t H) { return iso_ws_bytes(B, T, H); }

}  // extern "C"

namespace kdn {
namespace {
// Launches of the isotropic gain over B streams of the [.,T,H] rows: a
// fixed-length batch (tok = null, stream b = rows b*T ..) or a packed batch
// (tok = the sequences' token offsets, B = their count, Tgrid = the longest).
// phases: kIsoMaps (the segment maps, and their composition into `total`
// when given), kIsoFinish (the apply pass from the maps in the workspace).
constexpr int kIsoMaps = 1, kIsoFinish = 2, kIsoAll = 3;

int iso_fwd(const char* what, const float* a, const float* omega, const float* r, const float* init_prec,
            const float* init_cov, float* gain, float* p_prev, float* p_final, int64_t B, int64_t T, int64_t Tgrid,
            int64_t H, float s, const int* tok, void* workspace, size_t workspace_bytes, cudaStream_t st,
            int phases = kIsoAll, float* total = nullptr) {
  dim3 grid;
  if (int rc = iso_grid(what, B, Tgrid, H, workspace, workspace_bytes, &grid)) return rc;
  const IsoWs ws = iso_ws(workspace, (int)B, (int)grid.x, (int)H);
  if ((phases & kIsoMaps) && Tgrid > 0) {
    iso_gain_fwd_maps_kernel<<<grid, 32 * kIsoWarps, 0, st>>>(a, omega, r, ws, (int)T, (int)H, s, tok);
    if (int rc = check_launch("iso_gain_fwd_maps_kernel")) return rc;
    if (total) {
      iso_gain_fwd_total_kernel<<<(unsigned)((B * H + 127) / 128), 128, 0, st>>>(
          ws, reinterpret_cast<float4*>(total), (int)grid.x, (int)B, (int)H);
      if (int rc = check_launch("iso_gain_fwd_total_kernel")) return rc;
    }
  }
  if (!(phases & kIsoFinish)) return KDN_OK;
  iso_gain_fwd_apply_kernel<<<grid, 32 * kIsoWarps, 0, st>>>(a, omega, r, init_prec, init_cov, ws, gain, p_prev,
                                                            p_final, (int)T, (int)H, s, tok);
  return check_launch("iso_gain_fwd_apply_kernel");
}

int iso_bwd(const char* what, const float* a, const float* omega, const float* r, const float* init_prec,
            const float* init_cov, const float* dgain, const float* p_prev, const float* d_final_cov, float* da,
            float* domega, float* dr, float* dinit, float* d_init_cov, int64_t B, int64_t T, int64_t Tgrid, int64_t H,
            float s, const int* tok, void* workspace, size_t workspace_bytes, cudaStream_t st, int phases = kIsoAll,
            float* total = nullptr) {
  dim3 grid;
  if (int rc = iso_grid(what, B, Tgrid, H, workspace, workspace_bytes, &grid)) return rc;
  const IsoWs ws = iso_ws(workspace, (int)B, (int)grid.x, (int)H);
  if ((phases & kIsoMaps) && Tgrid > 0) {
    iso_gain_bwd_maps_kernel<<<grid, 32 * kIsoWarps, 0, st>>>(a, omega, r, dgain, p_prev, ws, (int)T, (int)H, s, tok);
    if (int rc = check_launch("iso_gain_bwd_maps_kernel")) return rc;
    if (total) {
      iso_gain_bwd_total_kernel<<<(unsigned)((B * H + 127) / 128), 128, 0, st>>>(
          ws, reinterpret_cast<float2*>(total), (int)grid.x, (int)B, (int)H);
      if (int rc = check_launch("iso_gain_bwd_total_kernel")) return rc;
    }
  }
  if (!(phases & kIsoFinish)) return KDN_OK;
  if (cudaMemsetAsync(dinit, 0, sizeof(float) * H, st) != cudaSuccess) return check_launch("memset d_initial_precision");
  iso_gain_bwd_apply_kernel<<<grid, 32 * kIsoWarps, 0, st>>>(a, omega, r, init_prec, dgain, p_prev, d_final_cov,
                                                            init_cov != nullptr, d_init_cov, ws, da, domega, dr,
                                                            dinit, (int)T, (int)H, s, tok);
  return check_launch("iso_gain_bwd_apply_kernel");
}
}  // namespace
}  // namespace kdn

extern "C" {

int kdn_iso_gain_fwd(const float* a, const float* omega, const float* r, const float* init_prec,
                     const float* init_cov, float* gain, float* p_prev, float* p_final, int64_t B, int64_t T,
                     int64_t H, float s, void* workspace, size_t workspace_bytes, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T < 0 || !a || !omega || !r || !init_prec || !gain)
    return set_error(KDN_ERR_INVALID, "kdn_iso_gain_fwd: invalid arguments");
  return iso_fwd("kdn_iso_gain_fwd", a, omega, r, init_prec, init_cov, gain, p_prev, p_final, B, T, T, H, s, nullptr,
                 workspace, workspace_bytes, (cudaStream_t)stream);
}

int kdn_iso_gain_bwd(const float* a, const float* omega, const float* r, const float* init_prec,
                     const float* init_cov, const float* dgain, const float* p_prev, const float* d_final_cov,
                     float* da, float* domega, float* dr, float* dinit, float* d_init_cov, int64_t B, int64_t T,
                     int64_t H, float s, void* workspace, size_t workspace_bytes, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T < 0 || !a || !omega || !r || !init_prec || !dgain || !da || !domega || !dr || !dinit ||
      (T > 0 && !p_prev))
    return set_error(KDN_ERR_INVALID, "kdn_iso_gain_bwd: invalid arguments");
  return iso_bwd("kdn_iso_gain_bwd", a, omega, r, init_prec, init_cov, dgain, p_prev, d_final_cov, da, domega, dr,
                 dinit, d_init_cov, B, T, T, H, s, nullptr, workspace, workspace_bytes, (cudaStream_t)stream);
}

int kdn_iso_gain_fwd_maps(const float* a, const float* omega, const float* r, float* total_map, int64_t B, int64_t T,
                          int64_t H, float s, void* workspace, size_t workspace_bytes, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !a || !omega || !r || !total_map)
    return set_error(KDN_ERR_INVALID, "kdn_iso_gain_fwd_maps: invalid arguments");
  return iso_fwd("kdn_iso_gain_fwd_maps", a, omega, r, nullptr, nullptr, nullptr, nullptr, nullptr, B, T, T, H, s,
                 nullptr, workspace, workspace_bytes, (cudaStream_t)stream, kIsoMaps, total_map);
}

int kdn_iso_gain_fwd_finish(const float* a, const float* omega, const float* r, const float* init_prec,
                            const float* init_cov, float* gain, float* p_prev, float* p_final, int64_t B, int64_t T,
                            int64_t H, float s, void* workspace, size_t workspace_bytes, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !a || !omega || !r || !init_prec || !gain)
    return set_error(KDN_ERR_INVALID, "kdn_iso_gain_fwd_finish: invalid arguments");
  return iso_fwd("kdn_iso_gain_fwd_finish", a, omega, r, init_prec, init_cov, gain, p_prev, p_final, B, T, T, H, s,
                 nullptr, workspace, workspace_bytes, (cudaStream_t)stream, kIsoFinish);
}

int kdn_iso_gain_bwd_maps(const float* a, const float* omega, const float* r, const float* dgain, const float* p_prev,
                          float* total_adjoint, int64_t B, int64_t T, int64_t H, float s, void* workspace,
                          size_t workspace_bytes, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !a || !omega || !r || !dgain || !p_prev || !total_adjoint)
    return set_error(KDN_ERR_INVALID, "kdn_iso_gain_bwd_maps: invalid arguments");
  return iso_bwd("kdn_iso_gain_bwd_maps", a, omega, r, nullptr, nullptr, dgain, p_prev, nullptr, nullptr, nullptr,
                 nullptr, nullptr, nullptr, B, T, T, H, s, nullptr, workspace, workspace_bytes, (cudaStream_t)stream,
                 kIsoMaps, total_adjoint);
}

int kdn_iso_gain_bwd_finish(const float* a, const float* omega, const float* r, const float* init_prec,
                            const float* init_cov, const float* dgain, const float* p_prev, const float* d_final_cov,
                            float* da, float* domega, float* dr, float* dinit, float* d_init_cov, int64_t B, int64_t T,
                            int64_t H, float s, void* workspace, size_t workspace_bytes, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !a || !omega || !r || !init_prec || !dgain || !p_prev || !da || !domega ||
      !dr || !dinit)
    return set_error(KDN_ERR_INVALID, "kdn_iso_gain_bwd_finish: invalid arguments");
  return iso_bwd("kdn_iso_gain_bwd_finish", a, omega, r, init_prec, init_cov, dgain, p_prev, d_final_cov, da, domega,
                 dr, dinit, d_init_cov, B, T, T, H, s, nullptr, workspace, workspace_bytes, (cudaStream_t)stream,
                 kIsoFinish);
}

size_t kdn_iso_gain_varlen_workspace_bytes(int64_t num_seqs, int64_t max_seq_len, int64_t H) {
  return iso_ws_bytes(num_seqs, max_seq_len, H);
}

int kdn_iso_gain_fwd_varlen(const float* a, const float* omega, const float* r, const float* init_prec,
                            const float* init_cov, float* gain, float* p_prev, float* p_final, int64_t T, int64_t H,
                            float s, const int32_t* varlen_table, int64_t num_seqs, int64_t max_seq_len,
                            void* workspace, size_t workspace_bytes, kdn_stream_t stream) {
  if (H <= 0 || T <= 0 || !a || !omega || !r || !init_prec || !gain || !varlen_table || num_seqs <= 0 ||
      max_seq_len <= 0 || max_seq_len > T)
    return set_error(KDN_ERR_INVALID, "kdn_iso_gain_fwd_varlen: invalid arguments");
  return iso_fwd("kdn_iso_gain_fwd_varlen", a, omega, r, init_prec, init_cov, gain, p_prev, p_final, num_seqs, T,
                 max_seq_len, H, s, varlen_table, workspace, workspace_bytes, (cudaStream_t)stream);
}

int kdn_iso_gain_bwd_varlen(const float* a, const float* omega, const float* r, const float* init_prec,
                            const float* init_cov, const float* dgain, const float* p_prev, const float* d_final_cov,
                            float* da, float* domega, float* dr, float* dinit, float* d_init_cov, int64_t T, int64_t H,
                            float s, const int32_t* varlen_table, int64_t num_seqs, int64_t max_seq_len,
                            void* workspace, size_t workspace_bytes, kdn_stream_t stream) {
  if (H <= 0 || T <= 0 || !a || !omega || !r || !init_prec || !dgain || !p_prev || !da || !domega || !dr ||
      !dinit || !varlen_table || num_seqs <= 0 || max_seq_len <= 0 || max_seq_len > T)
    return set_error(KDN_ERR_INVALID, "kdn_iso_gain_bwd_varlen: invalid arguments");
  return iso_bwd("kdn_iso_gain_bwd_varlen", a, omega, r, init_prec, init_cov, dgain, p_prev, d_final_cov, da, domega,
                 dr, dinit, d_init_cov, num_seqs, T, max_seq_len, H, s, varlen_table, workspace, workspace_bytes,
                 (cudaStream_t)stream);
}

// carry = [the covariance entering every 64-token segment, B*H*nseg*K |
//          the covariance before every token (p_prev), B*T*H*K]; the
// backward reads p_prev instead of re-running the recursion
int64_t kdn_diag_gain_carry_elems(int64_t B, int64_t T, int64_t H, int64_t K) {
  const int64_t nseg = (T + kDiagSeg - 1) / kDiagSeg;
  return B * H * nseg * K + B * T * H * K;
}

size_t kdn_diag_gain_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K) {
  const int64_t nseg = (T + kDiagSeg - 1) / kDiagSeg;
  const size_t maps = align_up(sizeof(float4) * B * H * nseg * K, 256);  // forward maps / backward maps+lam carry
  const size_t bwd = align_up(sizeof(float2) * B * H * nseg * K, 256) + align_up(sizeof(float) * B * H * nseg * K, 256) +
                     align_up(sizeof(float2) * B * H * T, 256);
  return maps > bwd ? maps : bwd;
}

}  // extern "C"

namespace kdn {
namespace {

// Launch helpers of the diagonal gain; the entry points validate first.
// Phases: forward = maps (per 64-token segment Moebius maps) -> carry ->
// emit; backward = maps (per segment adjoint maps, per-token reductions) ->
// carry -> emit.  The maps phase and the rest can be separate calls (the
// workspace keeps the maps in between), which sequence parallelism uses to
// compose the streams' maps across ranks before the carry.
struct DiagDims {
  int64_t B, T, H, K;
  int nseg;
  Varlen v;  // packed batch (B = 1): segments are the sequences' 64-token chunks
  // (sequence, head) streams of the carry kernels
  unsigned streams() const { return (unsigned)(v.on() ? (int64_t)v.n * H : B * H); }
  // the covariance before every token, after the segment carries in `carry`
  float* p_prev(float* carry) const { return carry + B * H * nseg * K; }
  const float* p_prev(const float* carry) const { return carry + B * H * nseg * K; }
};

int diag_dims(const char* what, int64_t B, int64_t T, int64_t H, int64_t K, DiagDims* d) {
  if (K != 64 && K != 128) return set_error(KDN_ERR_INVALID, "%s: K must be 64 or 128, got %lld", what, (long long)K);
  if (T > INT32_MAX || B * H > 65535) return set_error(KDN_ERR_INVALID, "%s: size too large", what);
  *d = DiagDims{B, T, H, K, (int)((T + kDiagSeg - 1) / kDiagSeg), Varlen{nullptr, nullptr, nullptr, nullptr, 0}};
  return KDN_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int K, bool V16>
void launch_fwd_map(dim3 grid, const DiagDims& d, const float* k, const float* alpha, const float* omega,
                    const float* r, float4* maps, cudaStream_t st) {
  diag_gain_map_kernel<K, V16><<<grid, K, 0, st>>>(k, alpha, omega, r, maps, (int)d.T, (int)d.H, d.nseg, d.v);
}

int diag_fwd_maps(const DiagDims& d, const float* k, const float* alpha, const float* omega, const float* r,
                  float4* maps, cudaStream_t st) {
  dim3 grid((unsigned)d.nseg, (unsigned)(d.B * d.H));
  const bool v16 = aligned16(k) && aligned16(alpha) && aligned16(omega);
  auto f = d.K == 128 ? (v16 ? launch_fwd_map<128, true> : launch_fwd_map<128, false>)
                      : (v16 ? launch_fwd_map<64, true> : launch_fwd_map<64, false>);
  f(grid, d, k, alpha, omega, r, maps, st);
  return check_launch("diag_gain_map_kernel");
}

template <int K, bool V16>
void launch_fwd_emit(dim3 grid, const DiagDims& d, const float* k, const float* alpha, const float* omega,
                     const float* r, float* carry, float* kappa, cudaStream_t st) {
  diag_gain_emit_kernel<K, V16><<<grid, K, 0, st>>>(k, alpha, omega, r, carry, kappa, d.p_prev(carry), (int)d.T,
                                                    (int)d.H, d.nseg, d.v);
}

int diag_fwd_finish(const DiagDims& d, const float* k, const float* alpha, const float* omega, const float* r,
                    const float* init_prec, const float* init_cov, const float4* maps, float* kappa, float* carry,
                    float* p_final, cudaStream_t st) {
  dim3 grid((unsigned)d.nseg, (unsigned)(d.B * d.H));
  const unsigned sh = d.streams();
  if (d.K == 128)
    diag_gain_carry_kernel<128><<<sh, 128, 0, st>>>(maps, init_prec, init_cov, carry, p_final, (int)d.H, d.nseg, d.v);
  else
    diag_gain_carry_kernel<64><<<sh, 64, 0, st>>>(maps, init_prec, init_cov, carry, p_final, (int)d.H, d.nseg, d.v);
  const bool v16 = aligned16(k) && aligned16(alpha) && aligned16(omega);
  auto f = d.K == 128 ? (v16 ? launch_fwd_emit<128, true> : launch_fwd_emit<128, false>)
                      : (v16 ? launch_fwd_emit<64, true> : launch_fwd_emit<64, false>);
  f(grid, d, k, alpha, omega, r, carry, kappa, st);
  return check_launch("diag_gain_fwd kernels");
}

// backward workspace: [maps float2 | lam carry | per-token (D, G)]
struct DiagBwdWs {
  float2* maps;
  float* lam;
  float2* dg_tok;
};
DiagBwdWs diag_bwd_ws(const DiagDims& d, void* ws) {
  char* w = static_cast<char*>(ws);
  DiagBwdWs out;
  out.maps = reinterpret_cast<float2*>(w);
  w += align_up(sizeof(float2) * d.B * d.H * d.nseg * d.K, 256);
  out.lam = reinterpret_cast<float*>(w);
  w += align_up(sizeof(float) * d.B * d.H * d.nseg * d.K, 256);
  out.dg_tok = reinterpret_cast<float2*>(w);
  return out;
}

template <int K, bool V16>
void launch_bwd_map(dim3 grid, const DiagDims& d, const float* k, const float* alpha, const float* omega,
                    const float* r, const float* dkappa, const float* carry, const DiagBwdWs& w, cudaStream_t st) {
  diag_gain_bwd_map_kernel<K, V16><<<grid, K, 0, st>>>(k, alpha, omega, r, dkappa, d.p_prev(carry), w.maps, w.dg_tok,
                                                       (int)d.T, (int)d.H, d.nseg, d.v);
}

int diag_bwd_maps(const DiagDims& d, const float* k, const float* alpha, const float* omega, const float* r,
                  const float* dkappa, const float* carry, const DiagBwdWs& w, cudaStream_t st) {
  dim3 grid((unsigned)d.nseg, (unsigned)(d.B * d.H));
  const bool v16 = aligned16(k) && aligned16(alpha) && aligned16(omega) && aligned16(dkappa) &&
                   aligned16(d.p_prev(carry));
  auto f = d.K == 128 ? (v16 ? launch_bwd_map<128, true> : launch_bwd_map<128, false>)
                      : (v16 ? launch_bwd_map<64, true> : launch_bwd_map<64, false>);
  f(grid, d, k, alpha, omega, r, dkappa, carry, w, st);
  return check_launch("diag_gain_bwd_map_kernel");
}

template <int K, bool V16>
void launch_bwd_emit(dim3 grid, const DiagDims& d, const float* k, const float* alpha, const float* omega,
                     const float* r, const float* init_prec, const bf16* wr, const bf16* rr, const float* dkappa,
                     const float* carry, float* dk, float* dalpha, bf16* domega_raw, bf16* dr_raw, float* dmu,
                     float* d_init_cov, const DiagBwdWs& w, cudaStream_t st) {
  diag_gain_bwd_emit_kernel<K, V16><<<grid, K, 0, st>>>(k, alpha, omega, r, init_prec, wr, rr, dkappa,
                                                        d.p_prev(carry), w.lam, w.dg_tok, dk, dalpha, domega_raw,
                                                        dr_raw, dmu, d_init_cov, (int)d.T, (int)d.H, d.nseg, d.v);
}

int diag_bwd_finish(const DiagDims& d, const float* k, const float* alpha, const float* omega, const float* r,
                    const float* init_prec, const float* init_cov, const bf16* wr, const bf16* rr,
                    const float* dkappa, const float* carry, const float* d_final_cov, float* dk, float* dalpha,
                    bf16* domega_raw, bf16* dr_raw, float* dinit, float* d_init_cov, const DiagBwdWs& w,
                    cudaStream_t st) {
  if (dinit && cudaMemsetAsync(dinit, 0, sizeof(float) * d.H, st) != cudaSuccess)
    return check_launch("memset d_initial_precision");
  float* dmu = init_cov ? nullptr : dinit;  // with a carried-in covariance the prior gets no gradient here
  dim3 grid((unsigned)d.nseg, (unsigned)(d.B * d.H));
  const unsigned sh = d.streams();
  if (d.K == 128)
    diag_gain_bwd_carry_kernel<128><<<sh, 128, 0, st>>>(w.maps, d_final_cov, w.lam, (int)d.H, d.nseg, d.v);
  else
    diag_gain_bwd_carry_kernel<64><<<sh, 64, 0, st>>>(w.maps, d_final_cov, w.lam, (int)d.H, d.nseg, d.v);
  const bool v16 = aligned16(k) && aligned16(alpha) && aligned16(omega) && aligned16(dkappa) &&
                   aligned16(d.p_prev(carry)) && aligned16(wr);
  auto f = d.K == 128 ? (v16 ? launch_bwd_emit<128, true> : launch_bwd_emit<128, false>)
                      : (v16 ? launch_bwd_emit<64, true> : launch_bwd_emit<64, false>);
  f(grid, d, k, alpha, omega, r, init_prec, wr, rr, dkappa, carry, dk, dalpha, domega_raw, dr_raw, dmu, d_init_cov, w,
    st);
  return check_launch("diag_gain_bwd kernels");
}

}  // namespace
}  // namespace kdn

extern "C" {

int kdn_diag_gain_fwd(const float* k, const float* alpha, const float* omega, const float* r, const float* init_prec,
                      const float* init_cov, float* kappa, float* carry, float* p_final, int64_t B, int64_t T,
                      int64_t H, int64_t K, void* ws, size_t ws_bytes, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !k || !alpha || !omega || !r || !init_prec || !kappa || !carry)
    return set_error(KDN_ERR_INVALID, "kdn_diag_gain_fwd: invalid arguments");
  DiagDims d;
  if (int rc = diag_dims("kdn_diag_gain_fwd", B, T, H, K, &d)) return rc;
  if (ws_bytes < kdn_diag_gain_workspace_bytes(B, T, H, K) || !ws)
    return set_error(KDN_ERR_WORKSPACE, "kdn_diag_gain_fwd: workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  float4* maps = static_cast<float4*>(ws);
  if (int rc = diag_fwd_maps(d, k, alpha, omega, r, maps, st)) return rc;
  return diag_fwd_finish(d, k, alpha, omega, r, init_prec, init_cov, maps, kappa, carry, p_final, st);
}

int kdn_diag_gain_fwd_maps(const float* k, const float* alpha, const float* omega, const float* r, float* total_map,
                           int64_t B, int64_t T, int64_t H, int64_t K, void* ws, size_t ws_bytes,
                           kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !k || !alpha || !omega || !r || !total_map)
    return set_error(KDN_ERR_INVALID, "kdn_diag_gain_fwd_maps: invalid arguments");
  DiagDims d;
  if (int rc = diag_dims("kdn_diag_gain_fwd_maps", B, T, H, K, &d)) return rc;
  if (ws_bytes < kdn_diag_gain_workspace_bytes(B, T, H, K) || !ws)
    return set_error(KDN_ERR_WORKSPACE, "kdn_diag_gain_fwd_maps: workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  float4* maps = static_cast<float4*>(ws);
  if (int rc = diag_fwd_maps(d, k, alpha, omega, r, maps, st)) return rc;
  const unsigned bh = (unsigned)(B * H);
  if (K == 128)
    diag_gain_total_kernel<128><<<bh, 128, 0, st>>>(maps, reinterpret_cast<float4*>(total_map), d.nseg);
  else
    diag_gain_total_kernel<64><<<bh, 64, 0, st>>>(maps, reinterpret_cast<float4*>(total_map), d.nseg);
  return check_launch("diag_gain_total_kernel");
}

int kdn_diag_gain_fwd_finish(const float* k, const float* alpha, const float* omega, const float* r,
                             const float* init_prec, const float* init_cov, float* kappa, float* carry,
                             float* p_final, int64_t B, int64_t T, int64_t H, int64_t K, void* ws, size_t ws_bytes,
                             kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !k || !alpha || !omega || !r || !init_prec || !kappa || !carry)
    return set_error(KDN_ERR_INVALID, "kdn_diag_gain_fwd_finish: invalid arguments");
  DiagDims d;
  if (int rc = diag_dims("kdn_diag_gain_fwd_finish", B, T, H, K, &d)) return rc;
  if (ws_bytes < kdn_diag_gain_workspace_bytes(B, T, H, K) || !ws)
    return set_error(KDN_ERR_WORKSPACE, "kdn_diag_gain_fwd_finish: workspace too small");
  return diag_fwd_finish(d, k, alpha, omega, r, init_prec, init_cov, static_cast<const float4*>(ws), kappa, carry,
                         p_final, (cudaStream_t)stream);
}

int kdn_diag_gain_fwd_noalloc(const float* k, const float* alpha, const float* omega, const float* r,
                              const float* init_prec, float* kappa, float* carry, float* p_final, int64_t B,
                              int64_t T, int64_t H, int64_t K, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !k || !alpha || !omega || !r || !init_prec || !kappa || !carry)
    return set_error(KDN_ERR_INVALID, "kdn_diag_gain_fwd_noalloc: invalid arguments");
  DiagDims d;
  if (int rc = diag_dims("kdn_diag_gain_fwd_noalloc", B, T, H, K, &d)) return rc;
  if (B * H * d.nseg * K > kNoAllocMapEntries)
    return set_error(KDN_ERR_INVALID,
                     "kdn_diag_gain_fwd_noalloc: B*H*ceil(T/64)*K = %lld exceeds the static scratch of %lld entries; "
                     "use kdn_diag_gain_fwd with caller workspace",
                     (long long)(B * H * d.nseg * K), (long long)kNoAllocMapEntries);
  float4* maps = nullptr;
  int rc = noalloc_maps(&maps);
  if (rc != KDN_OK) return rc;
  // Every map entry is written by diag_gain_map_kernel before the carry
  // kernel reads it, so the scratch needs no clearing between calls.
  cudaStream_t st = (cudaStream_t)stream;
  if ((rc = diag_fwd_maps(d, k, alpha, omega, r, maps, st))) return rc;
  return diag_fwd_finish(d, k, alpha, omega, r, init_prec, nullptr, maps, kappa, carry, p_final, st);
}

int kdn_diag_gain_bwd(const float* k, const float* alpha, const float* omega, const float* r, const float* init_prec,
                      const float* init_cov, const void* omega_raw, const void* r_raw, const float* dkappa,
                      const float* carry, const float* d_final_cov, float* dk, float* dalpha, void* domega_raw,
                      void* dr_raw, float* dinit, float* d_init_cov, int64_t B, int64_t T, int64_t H, int64_t K,
                      void* ws, size_t ws_bytes, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !k || !alpha || !omega || !r || !init_prec || !omega_raw || !r_raw || !dkappa ||
      !carry || !dk || !dalpha || !domega_raw || !dr_raw)
    return set_error(KDN_ERR_INVALID, "kdn_diag_gain_bwd: invalid arguments");
  DiagDims d;
  if (int rc = diag_dims("kdn_diag_gain_bwd", B, T, H, K, &d)) return rc;
  if (ws_bytes < kdn_diag_gain_workspace_bytes(B, T, H, K) || !ws)
    return set_error(KDN_ERR_WORKSPACE, "kdn_diag_gain_bwd: workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  const DiagBwdWs w = diag_bwd_ws(d, ws);
  if (int rc = diag_bwd_maps(d, k, alpha, omega, r, dkappa, carry, w, st)) return rc;
  return diag_bwd_finish(d, k, alpha, omega, r, init_prec, init_cov, static_cast<const bf16*>(omega_raw),
                         static_cast<const bf16*>(r_raw), dkappa, carry, d_final_cov, dk, dalpha,
                         static_cast<bf16*>(domega_raw), static_cast<bf16*>(dr_raw), dinit, d_init_cov, w, st);
}

int kdn_diag_gain_bwd_maps(const float* k, const float* alpha, const float* omega, const float* r,
                           const float* dkappa, const float* carry, float* total_adjoint, int64_t B, int64_t T,
                           int64_t H, int64_t K, void* ws, size_t ws_bytes, kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !k || !alpha || !omega || !r || !dkappa || !carry || !total_adjoint)
    return set_error(KDN_ERR_INVALID, "kdn_diag_gain_bwd_maps: invalid arguments");
  DiagDims d;
  if (int rc = diag_dims("kdn_diag_gain_bwd_maps", B, T, H, K, &d)) return rc;
  if (ws_bytes < kdn_diag_gain_workspace_bytes(B, T, H, K) || !ws)
    return set_error(KDN_ERR_WORKSPACE, "kdn_diag_gain_bwd_maps: workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  const DiagBwdWs w = diag_bwd_ws(d, ws);
  if (int rc = diag_bwd_maps(d, k, alpha, omega, r, dkappa, carry, w, st)) return rc;
  const unsigned bh = (unsigned)(B * H);
  if (K == 128)
    diag_gain_bwd_total_kernel<128><<<bh, 128, 0, st>>>(w.maps, reinterpret_cast<float2*>(total_adjoint), d.nseg);
  else
    diag_gain_bwd_total_kernel<64><<<bh, 64, 0, st>>>(w.maps, reinterpret_cast<float2*>(total_adjoint), d.nseg);
  return check_launch("diag_gain_bwd_total_kernel");
}

int kdn_diag_gain_bwd_finish(const float* k, const float* alpha, const float* omega, const float* r,
                             const float* init_prec, const float* init_cov, const void* omega_raw, const void* r_raw,
                             const float* dkappa, const float* carry, const float* d_final_cov, float* dk,
                             float* dalpha, void* domega_raw, void* dr_raw, float* dinit, float* d_init_cov,
                             int64_t B, int64_t T, int64_t H, int64_t K, void* ws, size_t ws_bytes,
                             kdn_stream_t stream) {
  if (B <= 0 || H <= 0 || T <= 0 || !k || !alpha || !omega || !r || !init_prec || !omega_raw || !r_raw || !dkappa ||
      !carry || !dk || !dalpha || !domega_raw || !dr_raw)
    return set_error(KDN_ERR_INVALID, "kdn_diag_gain_bwd_finish: invalid arguments");
  DiagDims d;
  if (int rc = diag_dims("kdn_diag_gain_bwd_finish", B, T, H, K, &d)) return rc;
  if (ws_bytes < kdn_diag_gain_workspace_bytes(B, T, H, K) || !ws)
    return set_error(KDN_ERR_WORKSPACE, "kdn_diag_gain_bwd_finish: workspace too small");
  return diag_bwd_finish(d, k, alpha, omega, r, init_prec, init_cov, static_cast<const bf16*>(omega_raw),
                         static_cast<const bf16*>(r_raw), dkappa, carry, d_final_cov, dk, dalpha,
                         static_cast<bf16*>(domega_raw), static_cast<bf16*>(dr_raw), dinit, d_init_cov,
                         diag_bwd_ws(d, ws), (cudaStream_t)stream);
}

int64_t kdn_diag_gain_varlen_carry_elems(int64_t T, int64_t H, int64_t K, int64_t num_chunks) {
  return T > 0 && H > 0 && K > 0 && num_chunks > 0 ? H * num_chunks * K + T * H * K : 0;
}

size_t kdn_diag_gain_varlen_workspace_bytes(int64_t T, int64_t H, int64_t K, int64_t num_chunks) {
  if (T <= 0 || H <= 0 || K <= 0 || num_chunks <= 0) return 0;
  const size_t maps = align_up(sizeof(float4) * H * num_chunks * K, 256);
  const size_t bwd = align_up(sizeof(float2) * H * num_chunks * K, 256) + align_up(sizeof(float) * H * num_chunks * K, 256) +
                     align_up(sizeof(float2) * H * T, 256);
  return maps > bwd ? maps : bwd;
}

}  // extern "C"

namespace kdn {
namespace {
int diag_varlen_dims(const char* what, int64_t T, int64_t H, int64_t K, const int32_t* table, int64_t num_seqs,
                     int64_t num_chunks, void* ws, size_t ws_bytes, DiagDims* d) {
  if (!table || num_seqs <= 0 || num_chunks < num_seqs || num_chunks > INT32_MAX)
    return set_error(KDN_ERR_INVALID, "%s: a kdn_varlen_plan table, num_seqs > 0 and num_chunks required", what);
  if (int rc = diag_dims(what, 1, T, H, K, d)) return rc;
  if (num_chunks * kDiagSeg < T) return set_error(KDN_ERR_INVALID, "%s: num_chunks does not cover T", what);
  if (!ws || ws_bytes < kdn_diag_gain_varlen_workspace_bytes(T, H, K, num_chunks))
    return set_error(KDN_ERR_WORKSPACE, "%s: workspace too small", what);
  d->nseg = (int)num_chunks;
  d->v = varlen_view(table, num_seqs);
  return KDN_OK;
}
}  // namespace
}  // namespace kdn

extern "C" {

int kdn_diag_gain_fwd_varlen(const float* k, const float* alpha, const float* omega, const float* r,
                             const float* init_prec, const float* init_cov, float* kappa, float* carry,
                             float* p_final, int64_t T, int64_t H, int64_t K, const int32_t* varlen_table,
                             int64_t num_seqs, int64_t num_chunks, void* ws, size_t ws_bytes, kdn_stream_t stream) {
  if (H <= 0 || T <= 0 || !k || !alpha || !omega || !r || !init_prec || !kappa || !carry)
    return set_error(KDN_ERR_INVALID, "kdn_diag_gain_fwd_varlen: invalid arguments");
  DiagDims d;
  if (int rc = diag_varlen_dims("kdn_diag_gain_fwd_varlen", T, H, K, varlen_table, num_seqs, num_chunks, ws, ws_bytes,
                                &d))
    return rc;
  cudaStream_t st = (cudaStream_t)stream;
  float4* maps = static_cast<float4*>(ws);
  if (int rc = diag_fwd_maps(d, k, alpha, omega, r, maps, st)) return rc;
  return diag_fwd_finish(d, k, alpha, omega, r, init_prec, init_cov, maps, kappa, carry, p_final, st);
}

int kdn_diag_gain_bwd_varlen(const float* k, const float* alpha, const float* omega, const float* r,
                             const float* init_prec, const float* init_cov, const void* omega_raw, const void* r_raw,
                             const float* dkappa, const float* carry, const float* d_final_cov, float* dk,
                             float* dalpha, void* domega_raw, void* dr_raw, float* dinit, float* d_init_cov,
                             int64_t T, int64_t H, int64_t K, const int32_t* varlen_table, int64_t num_seqs,
                             int64_t num_chunks, void* ws, size_t ws_bytes, kdn_stream_t stream) {
  if (H <= 0 || T <= 0 || !k || !alpha || !omega || !r || !init_prec || !omega_raw || !r_raw || !dkappa || !carry ||
      !dk || !dalpha || !domega_raw || !dr_raw)
    return set_error(KDN_ERR_INVALID, "kdn_diag_gain_bwd_varlen: invalid arguments");
  DiagDims d;
  if (int rc = diag_varlen_dims("kdn_diag_gain_bwd_varlen", T, H, K, varlen_table, num_seqs, num_chunks, ws, ws_bytes,
                                &d))
    return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const DiagBwdWs w = diag_bwd_ws(d, ws);
  if (int rc = diag_bwd_maps(d, k, alpha, omega, r, dkappa, carry, w, st)) return rc;
  return diag_bwd_finish(d, k, alpha, omega, r, init_prec, init_cov, static_cast<const bf16*>(omega_raw),
                         static_cast<const bf16*>(r_raw), dkappa, carry, d_final_cov, dk, dalpha,
                         static_cast<bf16*>(domega_raw), static_cast<bf16*>(dr_raw), dinit, d_init_cov, w, st);
}

}  // extern "C"
