// Per-chunk building blocks of the chunked KDN memory scan, shared by the
// forward, reverse-state and chunk-parallel backward kernels.
//
// Math (one (b,h) stream, chunk of L <= C tokens, local index i, gates in
// base 2 with g the chunk-local inclusive prefix of log2(alpha)):
//
//   A[i,j] = sum_c k_ic kappa_jc 2^(g_ic - g_jc)      (j <  i)
//   Q[i,j] = sum_c q_ic kappa_jc 2^(g_ic - g_jc)      (j <= i)
//   T = (I + A)^-1,  delta = T v - T (k*2^g) S0,
//   o = scale [ (q*2^g) S0 + Q delta ],
//   S_end = Diag(2^g_L) S0 + (kappa * 2^(g_L - g))^T delta
//
// which is the tokenwise recurrence S = Diag(alpha)S + kappa (v - k^T Diag(alpha) S)^T
// (iso_kdn_naive.py:308-332, diag_kdn_naive.py:479-500) unrolled over a
// chunk.  The gate factor 2^(g_i - g_j) is split around a per-chunk
// reference rho (the gate at the chunk's middle row):
//   Kr = k 2^(g - rho),  Qr = q 2^(g - rho),  Kc = kappa 2^(rho - g)
// so A = Kr Kc^T and Q = Qr Kc^T are plain tensor-core products, and
//   k*2^g = Kr * fr,  q*2^g = Qr * fr,  kappa*2^(g_L-g) = Kc * fL
// with per-channel fr = 2^rho, fL = 2^(g_L - rho).  When some channel's gate
// moves more than kRngMax bits away from rho inside the chunk the factors
// could leave the fp32 range; such chunks take an exact path that evaluates
// A and Q (and, backward, their gradients) element by element with
// 2^(g_i - g_j) <= 1, and use rho_row = 0, rho_col = g_L for the operands.
#pragma once

#include "kdn_common.cuh"

namespace kdn {

constexpr int kKD = 128;  // key width
constexpr int kVD = 128;  // value width
constexpr int kBV = 64;   // value tile of the sequential kernels
constexpr float kRngMax = 100.f;

template <bool ISO_, int C_, class OpT_>
struct Cfg {
  static constexpr bool ISO = ISO_;
  static constexpr int C = C_;
  static constexpr int NB = C / 16;
  using OpT = OpT_;
  static constexpr bool F32 = std::is_same<OpT, float>::value;
  static constexpr int PAD = F32 ? 0 : 8;  // bf16 rows padded by 16 B against bank conflicts
  static constexpr int LDK = kKD + PAD;
  static constexpr int LDV = kBV + PAD;
  static constexpr int LDVF = kVD + PAD;
  static constexpr int LDC = C + PAD;
  static constexpr int LDA = C + 4;  // fp32 C x C scratch
  static constexpr int CG = ISO ? 64 : 32;  // gate-prefix restart of the boundary convention
  static_assert(C == CG, "internal chunk must equal the boundary gate chunk");
};

struct ScanParams {
  const bf16* q;
  const bf16* k;
  const bf16* v;
  const float* g;
  const float* beta;
  const float* kappa;
  const float* S0;
  void* o;
  float* ST;
  float* Tsave;  // [BH][NT][C][C]
  float* Qsave;  // [BH][NT][C][C]
  void* h;       // [BH][NT][KD][VD] OpT, chunk-start states
  void* dh;      // [BH][NT][KD][VD] OpT, chunk-end state adjoints
  const void* dO;
  const float* dST;
  float* dS0;
  bf16* dq;
  bf16* dk;
  bf16* dv;
  float* dg;
  float* dbeta;
  float* dkappa;
  char* dbg;  // fp32 precision: per-CTA global scratch standing in for shared memory
  size_t dbg_stride;
  int B, T, H, NT;
  float scale;
};

// Per-chunk views of the staging buffers.
template <class CF>
struct Chunk {
  using OpT = typename CF::OpT;
  // raw inputs
  bf16* q;
  bf16* k;
  float* g;
  float* kap;   // diag
  float* beta;  // iso, [C]
  // per-row / per-channel scalars
  float* rq;  // iso rstd of q rows
  float* rk;  // iso rstd of k rows
  float* fr;
  float* fL;
  float* gL;
  float* gmid;   // gate at the reference row, per channel
  float* glast;  // gate at the last valid row, per channel
  float* red;    // [32] scratch
  // operands
  OpT* Kr;
  OpT* Qr;
  OpT* Kc;
  int L;
  int m;
  bool fast;
};

__host__ __device__ constexpr size_t A128(size_t x) { return align_up(x, 128); }
__host__ __device__ constexpr size_t cmax(size_t a, size_t b) { return a > b ? a : b; }

// Per-row / per-channel scalars of a chunk: rq, rk [C]; fr, fL, gL, gmid,
// glast [KD]; red [32].
template <class CF>
__host__ __device__ constexpr size_t small_floats() {
  return 2 * CF::C + 5 * kKD + 32;
}
template <class CF>
__device__ __forceinline__ void bind_small(Chunk<CF>& ch, float* small) {
  ch.rq = small;
  ch.rk = small + CF::C;
  ch.fr = small + 2 * CF::C;
  ch.fL = ch.fr + kKD;
  ch.gL = ch.fL + kKD;
  ch.gmid = ch.gL + kKD;
  ch.glast = ch.gmid + kKD;
  ch.red = ch.glast + kKD;
}

// Load rows x cols bf16 (row stride src_ld elements) into an OpT buffer.
template <class CF>
__device__ __forceinline__ void load_tile_op(typename CF::OpT* dst, int ld, const bf16* src, size_t src_ld, int rows,
                                             int valid, int cols) {
  if constexpr (!CF::F32) {
    copy_rows<true>(dst, (size_t)ld * 2, src, src_ld * 2, rows, valid, cols * 2);
  } else {
    for (int e = threadIdx.x; e < rows * cols; e += blockDim.x) {
      const int i = e / cols, c = e - i * cols;
      dst[(size_t)i * ld + c] = i < valid ? __bfloat162float(src[i * src_ld + c]) : 0.f;
    }
  }
}

__device__ __forceinline__ size_t tok_row(const ScanParams& p, int b, int h, int t) {
  return ((size_t)b * p.T + t) * p.H + h;
}

// Issue the loads of a chunk's q, k, g (and kappa or beta) rows.
template <class CF>
__device__ __forceinline__ void load_raw(const Chunk<CF>& ch, const ScanParams& p, int b, int h, int t0, int L) {
  constexpr bool SM = !CF::F32;
  const size_t r0 = tok_row(p, b, h, t0);
  const size_t rs = (size_t)p.H;
  copy_rows<SM>(ch.q, kKD * 2, p.q + r0 * kKD, rs * kKD * 2, CF::C, L, kKD * 2);
  copy_rows<SM>(ch.k, kKD * 2, p.k + r0 * kKD, rs * kKD * 2, CF::C, L, kKD * 2);
  copy_rows<SM>(ch.g, kKD * 4, p.g + r0 * kKD, rs * kKD * 4, CF::C, L, kKD * 4);
  if constexpr (CF::ISO) {
    for (int i = threadIdx.x; i < CF::C; i += blockDim.x) ch.beta[i] = i < L ? p.beta[r0 + (size_t)i * rs] : 0.f;
  } else {
    copy_rows<SM>(ch.kap, kKD * 4, p.kappa + r0 * kKD, rs * kKD * 4, CF::C, L, kKD * 4);
  }
}

template <class CF>
__device__ __forceinline__ float kappa_at(const Chunk<CF>& ch, int i, int c) {
  if constexpr (CF::ISO) {
    return ch.beta[i] * ch.rk[i] * to_f(ch.k[i * kKD + c]);
  } else {
    return ch.kap[i * kKD + c];
  }
}
template <class CF>
__device__ __forceinline__ float khat_at(const Chunk<CF>& ch, int i, int c) {
  if constexpr (CF::ISO) {
    return ch.rk[i] * to_f(ch.k[i * kKD + c]);
  } else {
    return to_f(ch.k[i * kKD + c]);
  }
}
template <class CF>
__device__ __forceinline__ float qhat_at(const Chunk<CF>& ch, int i, int c) {
  if constexpr (CF::ISO) {
    return ch.rq[i] * to_f(ch.q[i * kKD + c]);
  } else {
    return to_f(ch.q[i * kKD + c]);
  }
}

// Gate references of a chunk: rho for the rows (Kr, Qr) and for the columns (Kc).
template <class CF>
__device__ __forceinline__ float rho_row(const Chunk<CF>& ch, int c) {
  return ch.fast ? ch.g[ch.m * kKD + c] : 0.f;
}
template <class CF>
__device__ __forceinline__ float rho_col(const Chunk<CF>& ch, int c) {
  return ch.g[(ch.fast ? ch.m : ch.L - 1) * kKD + c];
}

// Row norms (iso), range check, per-channel factors and the three gated
// operands.  The caller places the barrier that publishes them.
template <class CF>
__device__ void prep_chunk(Chunk<CF>& ch) {
  constexpr int C = CF::C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int L = ch.L;
  ch.m = L >= C ? C / 2 : (((L - 1) / 2) & ~15);
  if constexpr (CF::ISO) {
    for (int row = warp; row < 2 * C; row += nw) {
      const bf16* src = row < C ? ch.q + row * kKD : ch.k + (row - C) * kKD;
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < kKD / 32; ++j) {
        const float x = to_f(src[lane + 32 * j]);
        ss += x * x;
      }
      ss = warp_sum(ss);
      if (lane == 0) (row < C ? ch.rq : ch.rk)[row % C] = rsqrtf(ss + 1e-6f);
    }
  }
  // range of the gate around the reference row
  float rng = 0.f;
  const float* gm = ch.g + ch.m * kKD;
  for (int e = threadIdx.x; e < L * kKD; e += blockDim.x) rng = fmaxf(rng, fabsf(ch.g[e] - gm[e % kKD]));
  rng = warp_max(rng);
  if (lane == 0) ch.red[warp] = rng;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < nw; ++w) tot = fmaxf(tot, ch.red[w]);
  ch.fast = tot <= kRngMax;
  for (int c = threadIdx.x; c < kKD; c += blockDim.x) {
    const float gl = ch.g[(L - 1) * kKD + c];
    const float rr = rho_row(ch, c), rc = rho_col(ch, c);
    ch.fr[c] = ex2(rr);
    ch.fL[c] = ex2(gl - rc);
    ch.gL[c] = ex2(gl);
    ch.gmid[c] = ch.g[ch.m * kKD + c];
    ch.glast[c] = gl;
  }
  using OpT = typename CF::OpT;
  for (int e = threadIdx.x; e < C * kKD; e += blockDim.x) {
    const int i = e / kKD, c = e - i * kKD;
    float kr = 0.f, qr = 0.f, kc = 0.f;
    if (i < L) {
      const float gi = ch.g[e];
      const float er = ex2(gi - rho_row(ch, c));
      const float ec = ex2(rho_col(ch, c) - gi);
      kr = khat_at(ch, i, c) * er;
      qr = qhat_at(ch, i, c) * er;
      kc = kappa_at(ch, i, c) * ec;
    }
    ch.Kr[i * CF::LDK + c] = from_f<OpT>(kr);
    ch.Qr[i * CF::LDK + c] = from_f<OpT>(qr);
    ch.Kc[i * CF::LDK + c] = from_f<OpT>(kc);
  }
}

// A (fp32, strictly lower) and Q (OpT operand, lower incl. diagonal; fp32
// copy to global when Qsave != nullptr).  Ends with a barrier.
template <class CF>
__device__ void chunk_scores(const Chunk<CF>& ch, float* sA, typename CF::OpT* sQ, float* Qsave) {
  constexpr int C = CF::C, NB = CF::NB;
  using OpT = typename CF::OpT;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (ch.fast) {
    constexpr int ntri = NB * (NB + 1) / 2;
    for (int job = warp; job < 2 * ntri; job += nw) {
      const bool isQ = job >= ntri;
      int tj = isQ ? job - ntri : job, I = 0;
      while (tj > I) {
        tj -= I + 1;
        ++I;
      }
      const int J = tj;
      float acc[1][2][4];
      zero_acc(acc);
      wgemm<1, 2, true, true>(acc, isQ ? ch.Qr : ch.Kr, CF::LDK, ch.Kc, CF::LDK, 16 * I, 16 * J, 0, kKD);
      for_acc<1, 2>(16 * I, 16 * J, [&](int, int nt, int e, int i, int j) {
        float x = acc[0][nt][e];
        if (isQ) {
          x = j <= i ? x : 0.f;
          sQ[i * CF::LDC + j] = from_f<OpT>(x);
          if (Qsave) Qsave[i * C + j] = x;
        } else {
          sA[i * CF::LDA + j] = j < i ? x : 0.f;
        }
      });
    }
    // blocks above the diagonal are structurally zero
    for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
      const int i = e / C, j = e - i * C;
      if ((j >> 4) > (i >> 4)) {
        sQ[i * CF::LDC + j] = from_f<OpT>(0.f);
        if (Qsave) Qsave[e] = 0.f;
      }
    }
  } else {
    // exact: 2^(g_i - g_j) <= 1 evaluated per element
    for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
      const int i = e / C, j = e - i * C;
      float a = 0.f, qq = 0.f;
      if (j <= i && i < ch.L) {
        for (int c = 0; c < kKD; ++c) {
          const float f = kappa_at(ch, j, c) * ex2(ch.g[i * kKD + c] - ch.g[j * kKD + c]);
          a = fmaf(khat_at(ch, i, c), f, a);
          qq = fmaf(qhat_at(ch, i, c), f, qq);
        }
      }
      sA[i * CF::LDA + j] = j < i ? a : 0.f;
      sQ[i * CF::LDC + j] = from_f<OpT>(qq);
      if (Qsave) Qsave[i * C + j] = qq;
    }
  }
  __syncthreads();
}

// T = (I + A)^-1 for unit lower-triangular I + A (A strictly lower, fp32).
// Writes sT (fp32, ld LDA, upper zero) and its OpT copy; Tsave (fp32 global)
// when non-null.  sX: fp32 scratch of (NB-1)*256 floats.  Ends with a barrier.
template <class CF>
__device__ void chunk_solve(const float* sA, float* sT, typename CF::OpT* sTb, float* sX, float* Tsave) {
  constexpr int C = CF::C, NB = CF::NB, LDA = CF::LDA;
  using OpT = typename CF::OpT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // zero everything above the diagonal blocks
  for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
    const int i = e / C, j = e - i * C;
    if ((j >> 4) > (i >> 4)) sT[i * LDA + j] = 0.f;
  }
  // diagonal 16x16 blocks: one warp per block, one lane per column
  if (warp < NB && lane < 16) {
    const int o = warp * 16, j = lane;
    float col[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float x = (i == j) ? 1.f : 0.f;
      if (i > j) {
#pragma unroll
        for (int l = 0; l < 16; ++l)
          if (l >= j && l < i) x = fmaf(-sA[(o + i) * LDA + o + l], col[l], x);
      }
      col[i] = x;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) sT[(o + i) * LDA + o + j] = col[i];
  }
  __syncthreads();
  // off-diagonal blocks by distance d: T_IJ = -T_II sum_{K=J}^{I-1} A_IK T_KJ
  for (int d = 1; d < NB; ++d) {
    const int nblk = NB - d;
    for (int e = threadIdx.x; e < nblk * 256; e += blockDim.x) {
      const int J = e >> 8, I = J + d, r = (e >> 4) & 15, c = e & 15;
      float x = 0.f;
      for (int kk = J * 16; kk < I * 16; ++kk) x = fmaf(sA[(I * 16 + r) * LDA + kk], sT[kk * LDA + J * 16 + c], x);
      sX[e] = x;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nblk * 256; e += blockDim.x) {
      const int J = e >> 8, I = J + d, r = (e >> 4) & 15, c = e & 15;
      float x = 0.f;
      for (int l = 0; l <= r; ++l) x = fmaf(sT[(I * 16 + r) * LDA + I * 16 + l], sX[(J << 8) + l * 16 + c], x);
      sT[(I * 16 + r) * LDA + J * 16 + c] = -x;
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
    const int i = e / C, j = e - i * C;
    const float x = sT[i * LDA + j];
    sTb[i * CF::LDC + j] = from_f<OpT>(x);
    if (Tsave) Tsave[e] = x;
  }
  __syncthreads();
}

// Load a saved fp32 C x C matrix into an OpT operand buffer.
template <class CF>
__device__ __forceinline__ void load_cc(typename CF::OpT* dst, const float* src) {
  for (int e = threadIdx.x; e < CF::C * CF::C; e += blockDim.x) {
    const int i = e / CF::C, j = e - i * CF::C;
    dst[i * CF::LDC + j] = from_f<typename CF::OpT>(src[e]);
  }
}

}  // namespace kdn
