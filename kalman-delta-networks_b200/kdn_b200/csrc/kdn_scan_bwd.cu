// Backward of the chunked KDN memory scan.
//
// 1. scan_bwd_state_kernel (one CTA per (value tile, b*h), chunks in reverse):
//    carries the state adjoint dS in registers,
//        ddelta  = scale Q^T dO + Kc (fL*dS)
//        dS_prev = Diag(2^g_L) dS + Diag(fr) (scale Qr^T dO - W0^T ddelta)
//    and stores the chunk-end adjoint of every chunk (bf16) for step 2.
// 2. scan_bwd_chunk_kernel (one CTA per (chunk, b*h), all chunks in parallel):
//    with the saved chunk-start state S0 and the chunk-end adjoint dS it
//    rebuilds delta and ddelta and forms every input gradient of the chunk:
//        dQ = scale dO delta^T,  dT = ddelta v^T + dW0 Kr^T,
//        dA = -T^T dT T^T,  dv = T^T ddelta,  dW0 = -ddelta (fr S0)^T,
//        dQr = scale dO (fr S0)^T + dQ Kc,  dKr = T^T dW0 + dA Kc,
//        dKc = delta (fL dS)^T + dA^T Kr + dQ^T Qr,
//    then maps (dKr, dQr, dKc) back through the gate factors to dk, dq,
//    dkappa and the natural-log gate cotangent (before the reverse chunk
//    cumsum, iso_kdn_chunk.py:2180-2186), and for the isotropic variant
//    through kappa = beta k_hat and the L2 normalisation.
// Replaces _chunk_kda_bwd_precum (iso_kdn_chunk.py:2089-2187) and
// _DiagKdnMemoryFunction.backward (diag_kdn_chunk.py:3258-3312).
#include "kdn_scan.cuh"

namespace kdn {

// ---------------------------------------------------------------------------
// 1. reverse state-adjoint sweep
// ---------------------------------------------------------------------------
template <class CF>
struct StateLayout {
  static constexpr size_t sz = sizeof(typename CF::OpT);
  static constexpr int C = CF::C;
  static constexpr size_t q = 0;
  static constexpr size_t k = q + A128((size_t)C * kKD * 2);
  static constexpr size_t g = k + A128((size_t)C * kKD * 2);
  static constexpr size_t kap = g + A128((size_t)C * kKD * 4);
  static constexpr size_t dOst = kap + A128(CF::ISO ? (size_t)C * 4 : (size_t)C * kKD * 4);  // diag fp32 dO
  static constexpr size_t dO = dOst + A128(CF::ISO ? 16 : (size_t)C * kBV * 4);  // two buffers
  static constexpr size_t Tb = dO + 2 * A128((size_t)C * CF::LDV * sz);          // two buffers
  static constexpr size_t Qb = Tb + 2 * A128((size_t)C * CF::LDC * sz);          // two buffers
  static constexpr size_t Kr = Qb + 2 * A128((size_t)C * CF::LDC * sz);
  static constexpr size_t Qr = Kr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Kc = Qr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t W = Kc + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t DS = W + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t DD = DS + A128((size_t)kKD * CF::LDV * sz);
  static constexpr size_t small = DD + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t bytes = small + A128(small_floats<CF>() * 4);
};

template <class CF>
__device__ __forceinline__ void stage_dO(void* dst, const ScanParams& p, int b, int h, int t0, int L, int v0,
                                         int ld) {
  constexpr int C = CF::C;
  const size_t r0 = tok_row(p, b, h, t0) * kVD + v0;
  if constexpr (CF::ISO) {
    load_tile_op<CF>(static_cast<typename CF::OpT*>(dst), ld, static_cast<const bf16*>(p.dO) + r0,
                     (size_t)p.H * kVD, C, L, kBV);
  } else {
    copy_rows<!CF::F32>(dst, kBV * 4, static_cast<const float*>(p.dO) + r0, (size_t)p.H * kVD * 4, C, L, kBV * 4);
  }
}

// The diagonal variant's fp32 cotangent as the OpT operand, rounded to bf16
// like the reference does before its backward kernels (diag_kdn_chunk.py:3277).
template <class CF>
__device__ __forceinline__ void convert_dO(typename CF::OpT* dst, const float* st) {
  using OpT = typename CF::OpT;
  for (int e = threadIdx.x; e < CF::C * kBV / 2; e += blockDim.x) {
    const int i = (2 * e) / kBV, c = 2 * e - i * kBV;
    const float2 x = *reinterpret_cast<const float2*>(st + i * kBV + c);
    const float a = __bfloat162float(__float2bfloat16_rn(x.x)), b = __bfloat162float(__float2bfloat16_rn(x.y));
    st_pair(dst + i * CF::LDV + c, a, b);
  }
}

template <class CF>
__global__ void __launch_bounds__(256, 1) scan_bwd_state_kernel(ScanParams p) {
  using OpT = typename CF::OpT;
  using Lo = StateLayout<CF>;
  constexpr int C = CF::C;
  constexpr int NTW = C / 8;
  constexpr int NJW = kKD / (8 * NTW);
  constexpr int NTU = C / 16;
  constexpr int NJU = kBV / (8 * NTU);
  extern __shared__ __align__(128) char smem[];
  char* base = CF::F32 ? p.dbg + (size_t)(blockIdx.y * gridDim.x + blockIdx.x) * p.dbg_stride : smem;

  Chunk<CF> ch;
  ch.q = reinterpret_cast<bf16*>(base + Lo::q);
  ch.k = reinterpret_cast<bf16*>(base + Lo::k);
  ch.g = reinterpret_cast<float*>(base + Lo::g);
  ch.kap = reinterpret_cast<float*>(base + Lo::kap);
  ch.beta = ch.kap;
  ch.Kr = reinterpret_cast<OpT*>(base + Lo::Kr);
  ch.Qr = reinterpret_cast<OpT*>(base + Lo::Qr);
  ch.Kc = reinterpret_cast<OpT*>(base + Lo::Kc);
  bind_small(ch, reinterpret_cast<float*>(base + Lo::small));
  float* dOst = reinterpret_cast<float*>(base + Lo::dOst);
  constexpr size_t dO_stride = A128((size_t)C * CF::LDV * sizeof(OpT));
  constexpr size_t cc_stride = A128((size_t)C * CF::LDC * sizeof(OpT));
  auto sdO_buf = [&](int i) { return reinterpret_cast<OpT*>(base + Lo::dO + i * dO_stride); };
  auto sTb_buf = [&](int i) { return reinterpret_cast<OpT*>(base + Lo::Tb + i * cc_stride); };
  auto sQb_buf = [&](int i) { return reinterpret_cast<OpT*>(base + Lo::Qb + i * cc_stride); };
  OpT* sDS = reinterpret_cast<OpT*>(base + Lo::DS);
  OpT* sW = reinterpret_cast<OpT*>(base + Lo::W);
  OpT* sDD = reinterpret_cast<OpT*>(base + Lo::DD);

  const int vt = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int warp = threadIdx.x >> 5;
  const int v0 = vt * kBV;

  float dS[1][8][4];
  for_acc<1, 8>(16 * warp, 0, [&](int, int nt, int e, int row, int col) {
    dS[0][nt][e] = p.dST ? p.dST[((size_t)bh * kKD + row) * kVD + v0 + col] : 0.f;
  });

  auto issue_loads = [&](int c, int buf) {
    const int t0 = c * C, L = min(C, p.T - t0);
    const size_t cc = (size_t)bh * p.NT + c;
    load_raw(ch, p, b, h, t0, L);
    load_cc<CF>(sTb_buf(buf), static_cast<const OpT*>(p.Tsave) + cc * C * C);
    load_cc<CF>(sQb_buf(buf), static_cast<const OpT*>(p.Qsave) + cc * C * C);
    stage_dO<CF>(CF::ISO ? static_cast<void*>(sdO_buf(buf)) : static_cast<void*>(dOst), p, b, h, t0, L, v0, CF::LDV);
    if constexpr (!CF::F32) cp_async_commit();
  };
  issue_loads(p.NT - 1, 0);

  for (int c = p.NT - 1; c >= 0; --c) {
    const int buf = (p.NT - 1 - c) & 1;
    OpT* sTb = sTb_buf(buf);
    OpT* sQb = sQb_buf(buf);
    OpT* sdO = sdO_buf(buf);
    ch.L = min(C, p.T - c * C);
    if constexpr (!CF::F32) cp_async_wait_all();
    __syncthreads();
    prep_chunk(ch);
    if constexpr (!CF::ISO) convert_dO<CF>(sdO, dOst);
    __syncthreads();
    if (c > 0) issue_loads(c - 1, buf ^ 1);

    // W0 = T Kr; fL-scaled adjoint operand; chunk-end adjoint to HBM
    const int I = warp / NJW;
    {
      float acc[1][NTW][4];
      zero_acc(acc);
      wgemm<1, NTW, true, false>(acc, sTb, CF::LDC, ch.Kr, CF::LDK, 16 * I, (warp % NJW) * 8 * NTW, 0, 16 * (I + 1));
      store_acc(sW, CF::LDK, acc, 16 * I, (warp % NJW) * 8 * NTW);
    }
    OpT* dhdst = static_cast<OpT*>(p.dh) + ((size_t)bh * p.NT + c) * kKD * kVD;
    for_acc_pairs<1, 8>(dS, 16 * warp, 0, [&](int, int, int, int row, int col, float x0, float x1) {
      const float f = ch.fL[row];
      st_pair(sDS + row * CF::LDV + col, f * x0, f * x1);
      st_pair(dhdst + (size_t)row * kVD + v0 + col, x0, x1);
    });
    __syncthreads();

    // ddelta = scale Q^T dO + Kc (fL dS)
    const int Iu = warp / NJU, nu = (warp % NJU) * 8 * NTU;
    {
      float a1[1][NTU][4], a2[1][NTU][4];
      zero_acc(a1);
      zero_acc(a2);
      wgemm<1, NTU, false, false>(a1, sQb, CF::LDC, sdO, CF::LDV, 16 * Iu, nu, 16 * Iu, C);
      wgemm<1, NTU, true, false>(a2, ch.Kc, CF::LDK, sDS, CF::LDV, 16 * Iu, nu, 0, kKD);
#pragma unroll
      for (int nt = 0; nt < NTU; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) a1[0][nt][e] = p.scale * a1[0][nt][e] + a2[0][nt][e];
      store_acc(sDD, CF::LDV, a1, 16 * Iu, nu);
    }
    __syncthreads();

    // dS <- Diag(2^g_L) dS + Diag(fr) (scale Qr^T dO - W0^T ddelta)
    {
      float a1[1][8][4], a2[1][8][4];
      zero_acc(a1);
      zero_acc(a2);
      wgemm<1, 8, false, false>(a1, ch.Qr, CF::LDK, sdO, CF::LDV, 16 * warp, 0, 0, C);
      wgemm<1, 8, false, false>(a2, sW, CF::LDK, sDD, CF::LDV, 16 * warp, 0, 0, C);
      for_acc<1, 8>(16 * warp, 0, [&](int, int nt, int e, int row, int) {
        dS[0][nt][e] = ch.gL[row] * dS[0][nt][e] + ch.fr[row] * (p.scale * a1[0][nt][e] - a2[0][nt][e]);
      });
    }
  }
  if (p.dS0) {
    for_acc<1, 8>(16 * warp, 0, [&](int, int nt, int e, int row, int col) {
      p.dS0[((size_t)bh * kKD + row) * kVD + v0 + col] = dS[0][nt][e];
    });
  }
}

// ---------------------------------------------------------------------------
// 2. chunk-parallel gradients
// ---------------------------------------------------------------------------
template <class CF>
struct ChunkLayout {
  static constexpr size_t sz = sizeof(typename CF::OpT);
  static constexpr int C = CF::C;
  // raw inputs
  static constexpr size_t q = 0;
  static constexpr size_t k = q + A128((size_t)C * kKD * 2);
  static constexpr size_t g = k + A128((size_t)C * kKD * 2);
  static constexpr size_t kap = g + A128((size_t)C * kKD * 4);
  static constexpr size_t raw_end = kap + A128(CF::ISO ? (size_t)C * 4 : (size_t)C * kKD * 4);
  // value-half loop (aliases the raw inputs)
  static constexpr size_t v = 0;
  static constexpr size_t dO = v + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t Del = dO + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t DD = Del + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t S0 = DD + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t dS = S0 + A128((size_t)kKD * CF::LDV * sz);
  static constexpr size_t dOst = dS + A128((size_t)kKD * CF::LDV * sz);  // diag fp32 dO staging
  static constexpr size_t loop_end = dOst + A128(CF::ISO ? 16 : (size_t)C * kBV * 4);
  // after the loop (aliases again)
  static constexpr size_t dW = 0;
  static constexpr size_t dT = dW + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t X = dT + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t dA = X + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t dQ = dA + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t dAf = dQ + A128((size_t)C * CF::LDC * sz);  // fp32 copies for the exact path
  static constexpr size_t dQf = dAf + A128((size_t)C * C * 4);
  static constexpr size_t post_end = dQf + A128((size_t)C * C * 4);
  static constexpr size_t Kr = cmax(cmax(raw_end, loop_end), post_end);
  static constexpr size_t Qr = Kr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Kc = Qr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Tb = Kc + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Qb = Tb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t W = Qb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t small = W + A128((size_t)C * CF::LDK * sz);
  // small: chunk scalars, cfl[KD], cgl[KD], rows: dbeta, dotk, dotq [C]
  static constexpr size_t bytes = small + A128((small_floats<CF>() + 2 * kKD + 3 * C) * 4);
};

template <class CF>
__global__ void __launch_bounds__(512, 1) scan_bwd_chunk_kernel(ScanParams p) {
  using OpT = typename CF::OpT;
  using Lo = ChunkLayout<CF>;
  constexpr int C = CF::C, NB = CF::NB;
  constexpr int NTK = C / 16;             // C x 128 tiles: 16 x 8NTK per warp
  constexpr int NJK = kKD / (8 * NTK);
  constexpr int NTV = C / 32;             // C x 64 tiles: 16 x 8NTV per warp
  constexpr int NJV = kBV / (8 * NTV);
  constexpr int NTRI = NB * (NB + 1) / 2; // lower 16x16 tiles of C x C
  static_assert((C / 16) * NJK == 16 && (C / 16) * NJV == 16, "16 warps");
  extern __shared__ __align__(128) char smem[];
  char* base = CF::F32 ? p.dbg + (size_t)(blockIdx.y * gridDim.x + blockIdx.x) * p.dbg_stride : smem;

  Chunk<CF> ch;
  ch.q = reinterpret_cast<bf16*>(base + Lo::q);
  ch.k = reinterpret_cast<bf16*>(base + Lo::k);
  ch.g = reinterpret_cast<float*>(base + Lo::g);
  ch.kap = reinterpret_cast<float*>(base + Lo::kap);
  ch.beta = ch.kap;
  ch.Kr = reinterpret_cast<OpT*>(base + Lo::Kr);
  ch.Qr = reinterpret_cast<OpT*>(base + Lo::Qr);
  ch.Kc = reinterpret_cast<OpT*>(base + Lo::Kc);
  float* small = reinterpret_cast<float*>(base + Lo::small);
  bind_small(ch, small);
  float* cfl = small + small_floats<CF>();
  float* cgl = cfl + kKD;
  float* rbeta = cgl + kKD;
  float* rdotk = rbeta + C;
  float* rdotq = rdotk + C;
  OpT* sv = reinterpret_cast<OpT*>(base + Lo::v);
  OpT* sdO = reinterpret_cast<OpT*>(base + Lo::dO);
  OpT* sDel = reinterpret_cast<OpT*>(base + Lo::Del);
  OpT* sDD = reinterpret_cast<OpT*>(base + Lo::DD);
  OpT* sS0 = reinterpret_cast<OpT*>(base + Lo::S0);
  OpT* sdS = reinterpret_cast<OpT*>(base + Lo::dS);
  float* dOst = reinterpret_cast<float*>(base + Lo::dOst);
  OpT* sdW = reinterpret_cast<OpT*>(base + Lo::dW);
  OpT* sdT = reinterpret_cast<OpT*>(base + Lo::dT);
  OpT* sX = reinterpret_cast<OpT*>(base + Lo::X);
  OpT* sdA = reinterpret_cast<OpT*>(base + Lo::dA);
  OpT* sdQ = reinterpret_cast<OpT*>(base + Lo::dQ);
  float* sdAf = reinterpret_cast<float*>(base + Lo::dAf);
  float* sdQf = reinterpret_cast<float*>(base + Lo::dQf);
  OpT* sTb = reinterpret_cast<OpT*>(base + Lo::Tb);
  OpT* sQb = reinterpret_cast<OpT*>(base + Lo::Qb);
  OpT* sW = reinterpret_cast<OpT*>(base + Lo::W);

  const int c = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = c * C;
  const int L = min(C, p.T - t0);
  const size_t cc = (size_t)bh * p.NT + c;
  ch.L = L;

  load_raw(ch, p, b, h, t0, L);
  load_cc<CF>(sTb, static_cast<const OpT*>(p.Tsave) + cc * C * C);
  load_cc<CF>(sQb, static_cast<const OpT*>(p.Qsave) + cc * C * C);
  if constexpr (!CF::F32) {
    cp_async_commit();
    cp_async_wait_all();
  }
  __syncthreads();
  prep_chunk(ch);
  for (int e = threadIdx.x; e < 2 * kKD + 3 * C; e += blockDim.x) cfl[e] = 0.f;
  __syncthreads();

  // W0 = T Kr
  const int I = warp / NJK, n0 = (warp % NJK) * 8 * NTK;
  {
    float acc[1][NTK][4];
    zero_acc(acc);
    wgemm<1, NTK, true, false>(acc, sTb, CF::LDC, ch.Kr, CF::LDK, 16 * I, n0, 0, 16 * (I + 1));
    store_acc(sW, CF::LDK, acc, 16 * I, n0);
  }
  __syncthreads();

  // lower C x C tile owned by this warp (for dQ, dT, X, dA)
  int TI = 0, TJ = warp;
  while (TJ > TI) {
    TJ -= TI + 1;
    ++TI;
  }
  const bool own_tri = warp < NTRI;

  float aQr[1][NTK][4], aW[1][NTK][4], aKc[1][NTK][4];
  float aDQ[1][2][4], aDT[1][2][4];
  zero_acc(aQr);
  zero_acc(aW);
  zero_acc(aKc);
  zero_acc(aDQ);
  zero_acc(aDT);
  const int Iv = warp / NJV, nv = (warp % NJV) * 8 * NTV;
  const OpT* hsrc = static_cast<const OpT*>(p.h) + cc * kKD * kVD;
  const OpT* dhsrc = static_cast<const OpT*>(p.dh) + cc * kKD * kVD;

  for (int vh = 0; vh < kVD / kBV; ++vh) {
    const int v0 = vh * kBV;
    const size_t r0 = tok_row(p, b, h, t0);
    load_tile_op<CF>(sv, CF::LDV, p.v + r0 * kVD + v0, (size_t)p.H * kVD, C, L, kBV);
    if constexpr (CF::ISO) {
      load_tile_op<CF>(sdO, CF::LDV, static_cast<const bf16*>(p.dO) + r0 * kVD + v0, (size_t)p.H * kVD, C, L, kBV);
    } else {
      copy_rows<!CF::F32>(dOst, kBV * 4, static_cast<const float*>(p.dO) + r0 * kVD + v0, (size_t)p.H * kVD * 4, C, L,
                          kBV * 4);
    }
    copy_rows<!CF::F32>(sS0, CF::LDV * sizeof(OpT), hsrc + v0, kVD * sizeof(OpT), kKD, kKD, kBV * sizeof(OpT));
    copy_rows<!CF::F32>(sdS, CF::LDV * sizeof(OpT), dhsrc + v0, kVD * sizeof(OpT), kKD, kKD, kBV * sizeof(OpT));
    if constexpr (!CF::F32) {
      cp_async_commit();
      cp_async_wait_all();
    }
    __syncthreads();
    if constexpr (!CF::ISO) convert_dO<CF>(sdO, dOst);
    // S0' = fr S0, dS'' = fL dS, and cgl += sum_v S0' dS''  (4 threads per channel)
    {
      const int ch_ = threadIdx.x >> 2, part = threadIdx.x & 3;
      float acc = 0.f;
      if (ch_ < kKD) {
        const float fr = ch.fr[ch_], fl = ch.fL[ch_];
        for (int vv = part * (kBV / 4); vv < (part + 1) * (kBV / 4); ++vv) {
          const float s0 = fr * to_f(sS0[ch_ * CF::LDV + vv]);
          const float ds = fl * to_f(sdS[ch_ * CF::LDV + vv]);
          sS0[ch_ * CF::LDV + vv] = from_f<OpT>(s0);
          sdS[ch_ * CF::LDV + vv] = from_f<OpT>(ds);
          acc = fmaf(s0, ds, acc);
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (ch_ < kKD && part == 0) cgl[ch_] += acc;
    }
    __syncthreads();

    // delta = T v - W0 S0',  ddelta = scale Q^T dO + Kc dS''
    {
      float u[1][NTV][4], a[1][NTV][4];
      zero_acc(u);
      zero_acc(a);
      wgemm<1, NTV, true, false>(u, sTb, CF::LDC, sv, CF::LDV, 16 * Iv, nv, 0, 16 * (Iv + 1));
      wgemm<1, NTV, true, false>(a, sW, CF::LDK, sS0, CF::LDV, 16 * Iv, nv, 0, kKD);
      for_acc<1, NTV>(16 * Iv, nv, [&](int, int nt, int e, int row, int col) {
        sDel[row * CF::LDV + col] = from_f<OpT>(u[0][nt][e] - a[0][nt][e]);
      });
      zero_acc(u);
      zero_acc(a);
      wgemm<1, NTV, false, false>(u, sQb, CF::LDC, sdO, CF::LDV, 16 * Iv, nv, 16 * Iv, C);
      wgemm<1, NTV, true, false>(a, ch.Kc, CF::LDK, sdS, CF::LDV, 16 * Iv, nv, 0, kKD);
      for_acc<1, NTV>(16 * Iv, nv, [&](int, int nt, int e, int row, int col) {
        sDD[row * CF::LDV + col] = from_f<OpT>(p.scale * u[0][nt][e] + a[0][nt][e]);
      });
    }
    __syncthreads();

    // dv = T^T ddelta
    {
      float a[1][NTV][4];
      zero_acc(a);
      wgemm<1, NTV, false, false>(a, sTb, CF::LDC, sDD, CF::LDV, 16 * Iv, nv, 16 * Iv, C);
      for_acc<1, NTV>(16 * Iv, nv, [&](int, int nt, int e, int row, int col) {
        if (row < L) p.dv[tok_row(p, b, h, t0 + row) * kVD + v0 + col] = __float2bfloat16_rn(a[0][nt][e]);
      });
    }
    // value-contracted accumulations
    wgemm<1, NTK, true, true>(aQr, sdO, CF::LDV, sS0, CF::LDV, 16 * I, n0, 0, kBV);
    wgemm<1, NTK, true, true>(aW, sDD, CF::LDV, sS0, CF::LDV, 16 * I, n0, 0, kBV);
    wgemm<1, NTK, true, true>(aKc, sDel, CF::LDV, sdS, CF::LDV, 16 * I, n0, 0, kBV);
    if (own_tri) {
      wgemm<1, 2, true, true>(aDQ, sdO, CF::LDV, sDel, CF::LDV, 16 * TI, 16 * TJ, 0, kBV);
      wgemm<1, 2, true, true>(aDT, sDD, CF::LDV, sv, CF::LDV, 16 * TI, 16 * TJ, 0, kBV);
    }
    __syncthreads();
  }

  // cfl[c] = sum_j Kc_jc (delta dS''^T)_jc: the fL cotangent of the last row
  {
    float part[NTK][2];
#pragma unroll
    for (int nt = 0; nt < NTK; ++nt) part[nt][0] = part[nt][1] = 0.f;
    for_acc<1, NTK>(16 * I, n0, [&](int, int nt, int e, int row, int col) {
      part[nt][e & 1] += to_f(ch.Kc[row * CF::LDK + col]) * aKc[0][nt][e];
    });
#pragma unroll
    for (int nt = 0; nt < NTK; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float x = part[nt][j];
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        x += __shfl_xor_sync(0xffffffffu, x, 16);
        if (lane < 4) atomicAdd(&cfl[n0 + nt * 8 + 2 * lane + j], x);
      }
  }

  // post-loop buffers (alias the loop buffers)
#pragma unroll
  for (int nt = 0; nt < NTK; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      aQr[0][nt][e] *= p.scale;
      aW[0][nt][e] = -aW[0][nt][e];
    }
  store_acc(sdW, CF::LDK, aW, 16 * I, n0);
  for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
    const int i = e / C, j = e - i * C;
    if ((j >> 4) > (i >> 4)) {
      sdT[i * CF::LDC + j] = from_f<OpT>(0.f);
      sX[i * CF::LDC + j] = from_f<OpT>(0.f);
      sdA[i * CF::LDC + j] = from_f<OpT>(0.f);
      sdQ[i * CF::LDC + j] = from_f<OpT>(0.f);
      sdAf[e] = 0.f;
      sdQf[e] = 0.f;
    }
  }
  if (own_tri) {
    for_acc<1, 2>(16 * TI, 16 * TJ, [&](int, int nt, int e, int row, int col) {
      const float x = col <= row ? p.scale * aDQ[0][nt][e] : 0.f;
      sdQ[row * CF::LDC + col] = from_f<OpT>(x);
      sdQf[row * C + col] = x;
    });
  }
  __syncthreads();

  // dKr = T^T dW0;  dT += dW0 Kr^T
  float aKr[1][NTK][4];
  zero_acc(aKr);
  wgemm<1, NTK, false, false>(aKr, sTb, CF::LDC, sdW, CF::LDK, 16 * I, n0, 16 * I, C);
  if (own_tri) {
    wgemm<1, 2, true, true>(aDT, sdW, CF::LDK, ch.Kr, CF::LDK, 16 * TI, 16 * TJ, 0, kKD);
    for_acc<1, 2>(16 * TI, 16 * TJ, [&](int, int nt, int e, int row, int col) {
      sdT[row * CF::LDC + col] = from_f<OpT>(col < row ? aDT[0][nt][e] : 0.f);
    });
  }
  __syncthreads();
  // X = dT T^T (lower tiles), then dA = -T^T X (strictly lower)
  if (own_tri) {
    float x[1][2][4];
    zero_acc(x);
    wgemm<1, 2, true, true>(x, sdT, CF::LDC, sTb, CF::LDC, 16 * TI, 16 * TJ, 0, 16 * (TJ + 1));
    store_acc(sX, CF::LDC, x, 16 * TI, 16 * TJ);
  }
  __syncthreads();
  if (own_tri) {
    float x[1][2][4];
    zero_acc(x);
    wgemm<1, 2, false, false>(x, sTb, CF::LDC, sX, CF::LDC, 16 * TI, 16 * TJ, 16 * TI, C);
    for_acc<1, 2>(16 * TI, 16 * TJ, [&](int, int nt, int e, int row, int col) {
      const float y = col < row ? -x[0][nt][e] : 0.f;
      sdA[row * CF::LDC + col] = from_f<OpT>(y);
      sdAf[row * C + col] = y;
    });
  }
  __syncthreads();
  if (ch.fast) {
    wgemm<1, NTK, true, false>(aKr, sdA, CF::LDC, ch.Kc, CF::LDK, 16 * I, n0, 0, 16 * (I + 1));
    wgemm<1, NTK, true, false>(aQr, sdQ, CF::LDC, ch.Kc, CF::LDK, 16 * I, n0, 0, 16 * (I + 1));
    wgemm<1, NTK, false, false>(aKc, sdA, CF::LDC, ch.Kr, CF::LDK, 16 * I, n0, 16 * I, C);
    wgemm<1, NTK, false, false>(aKc, sdQ, CF::LDC, ch.Qr, CF::LDK, 16 * I, n0, 16 * I, C);
  }

  // map back through the gate factors
  float aG[1][NTK][4];
  float rsum[2] = {0.f, 0.f};  // iso: dbeta partials of rows g, g+8
  for_acc<1, NTK>(16 * I, n0, [&](int, int nt, int e, int row, int col) {
    aG[0][nt][e] = 0.f;
    if (row >= L) return;
    const size_t rowg = tok_row(p, b, h, t0 + row);
    const float gi = p.g[rowg * kKD + col];
    const float rr = ch.fast ? ch.gmid[col] : 0.f;
    const float rc = ch.fast ? ch.gmid[col] : ch.glast[col];
    const float er = ex2(gi - rr), ec = ex2(rc - gi);
    float kh, qh, kap;
    if constexpr (CF::ISO) {
      kh = ch.rk[row] * __bfloat162float(p.k[rowg * kKD + col]);
      qh = ch.rq[row] * __bfloat162float(p.q[rowg * kKD + col]);
      kap = p.beta[rowg] * kh;
    } else {
      kh = __bfloat162float(p.k[rowg * kKD + col]);
      qh = __bfloat162float(p.q[rowg * kKD + col]);
      kap = p.kappa[rowg * kKD + col];
    }
    float dkh = aKr[0][nt][e] * er, dqh = aQr[0][nt][e] * er, dkap = aKc[0][nt][e] * ec;
    float dG = aKr[0][nt][e] * kh * er + aQr[0][nt][e] * qh * er - aKc[0][nt][e] * kap * ec;
    if (row == L - 1) dG += cfl[col] + cgl[col] * ch.gL[col] / (ch.fr[col] * ch.fL[col]);
    if (!ch.fast) {
      // exact gate factors for the score terms
      for (int j = 0; j < L; ++j) {
        const size_t rowj = tok_row(p, b, h, t0 + j);
        const float gj = p.g[rowj * kKD + col];
        float khj, qhj, kapj;
        if constexpr (CF::ISO) {
          khj = ch.rk[j] * __bfloat162float(p.k[rowj * kKD + col]);
          qhj = ch.rq[j] * __bfloat162float(p.q[rowj * kKD + col]);
          kapj = p.beta[rowj] * khj;
        } else {
          khj = __bfloat162float(p.k[rowj * kKD + col]);
          qhj = __bfloat162float(p.q[rowj * kKD + col]);
          kapj = p.kappa[rowj * kKD + col];
        }
        if (j <= row) {
          const float f = ex2(gi - gj);
          const float dAij = j < row ? sdAf[row * C + j] : 0.f;
          const float dQij = sdQf[row * C + j];
          dkh = fmaf(dAij * kapj, f, dkh);
          dqh = fmaf(dQij * kapj, f, dqh);
          dG = fmaf((dAij * kh + dQij * qh) * kapj, f, dG);
        }
        if (j >= row) {
          const float f = ex2(gj - gi);
          const float dAji = j > row ? sdAf[j * C + row] : 0.f;
          const float dQji = sdQf[j * C + row];
          const float w = (dAji * khj + dQji * qhj) * f;
          dkap += w;
          dG -= w * kap;
        }
      }
    }
    aG[0][nt][e] = dG;
    if constexpr (CF::ISO) {
      rsum[e >> 1] += dkap * kh;                 // dbeta_i = sum_c dkappa_ic k_hat_ic
      dkh += p.beta[rowg] * dkap;                // kappa = beta k_hat
    } else {
      p.dkappa[rowg * kKD + col] = dkap;
    }
    aKr[0][nt][e] = dkh;
    aQr[0][nt][e] = dqh;
    p.dg[rowg * kKD + col] = dG;
  });

  if constexpr (CF::ISO) {
    // row reductions: dbeta, <dk_hat, k_hat>, <dq_hat, q_hat>
    float dk_dot[2] = {0.f, 0.f}, dq_dot[2] = {0.f, 0.f};
    for_acc<1, NTK>(16 * I, n0, [&](int, int nt, int e, int row, int col) {
      if (row >= L) return;
      const size_t rowg = tok_row(p, b, h, t0 + row);
      const float kh = ch.rk[row] * __bfloat162float(p.k[rowg * kKD + col]);
      const float qh = ch.rq[row] * __bfloat162float(p.q[rowg * kKD + col]);
      dk_dot[e >> 1] += aKr[0][nt][e] * kh;
      dq_dot[e >> 1] += aQr[0][nt][e] * qh;
    });
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float x0 = rsum[j], x1 = dk_dot[j], x2 = dq_dot[j];
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        x0 += __shfl_xor_sync(0xffffffffu, x0, o);
        x1 += __shfl_xor_sync(0xffffffffu, x1, o);
        x2 += __shfl_xor_sync(0xffffffffu, x2, o);
      }
      if ((lane & 3) == 0) {
        const int row = 16 * I + (lane >> 2) + 8 * j;
        atomicAdd(&rbeta[row], x0);
        atomicAdd(&rdotk[row], x1);
        atomicAdd(&rdotq[row], x2);
      }
    }
    __syncthreads();
    for_acc<1, NTK>(16 * I, n0, [&](int, int nt, int e, int row, int col) {
      if (row >= L) return;
      const size_t rowg = tok_row(p, b, h, t0 + row);
      const float kh = ch.rk[row] * __bfloat162float(p.k[rowg * kKD + col]);
      const float qh = ch.rq[row] * __bfloat162float(p.q[rowg * kKD + col]);
      p.dk[rowg * kKD + col] = __float2bfloat16_rn(ch.rk[row] * (aKr[0][nt][e] - kh * rdotk[row]));
      p.dq[rowg * kKD + col] = __float2bfloat16_rn(ch.rq[row] * (aQr[0][nt][e] - qh * rdotq[row]));
    });
    for (int i = threadIdx.x; i < L; i += blockDim.x) p.dbeta[tok_row(p, b, h, t0 + i)] = rbeta[i];
  } else {
    for_acc<1, NTK>(16 * I, n0, [&](int, int nt, int e, int row, int col) {
      if (row >= L) return;
      const size_t rowg = tok_row(p, b, h, t0 + row);
      p.dk[rowg * kKD + col] = __float2bfloat16_rn(aKr[0][nt][e]);
      p.dq[rowg * kKD + col] = __float2bfloat16_rn(aQr[0][nt][e]);
    });
  }
  (void)aG;
}

// ---------------------------------------------------------------------------
template <class CF>
size_t state_bytes() {
  return StateLayout<CF>::bytes;
}
template <class CF>
size_t chunk_bytes() {
  return ChunkLayout<CF>::bytes;
}

template <class CF>
int launch_bwd(const ScanParams& p, cudaStream_t st) {
  const size_t s1 = CF::F32 ? 0 : StateLayout<CF>::bytes;
  const size_t s2 = CF::F32 ? 0 : ChunkLayout<CF>::bytes;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(scan_bwd_state_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s1) !=
        cudaSuccess)
      return check_launch("cudaFuncSetAttribute(scan_bwd_state_kernel)");
    if (cudaFuncSetAttribute(scan_bwd_chunk_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s2) !=
        cudaSuccess)
      return check_launch("cudaFuncSetAttribute(scan_bwd_chunk_kernel)");
    configured = true;
  }
  scan_bwd_state_kernel<CF><<<dim3(kVD / kBV, p.B * p.H), 256, s1, st>>>(p);
  int rc = check_launch("scan_bwd_state_kernel");
  if (rc != KDN_OK) return rc;
  scan_bwd_chunk_kernel<CF><<<dim3(p.NT, p.B * p.H), 512, s2, st>>>(p);
  return check_launch("scan_bwd_chunk_kernel");
}

template int launch_bwd<Cfg<true, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_bwd<Cfg<true, 64, float>>(const ScanParams&, cudaStream_t);
template int launch_bwd<Cfg<false, 32, bf16>>(const ScanParams&, cudaStream_t);
template int launch_bwd<Cfg<false, 32, float>>(const ScanParams&, cudaStream_t);
template size_t state_bytes<Cfg<true, 64, float>>();
template size_t state_bytes<Cfg<false, 32, float>>();
template size_t chunk_bytes<Cfg<true, 64, float>>();
template size_t chunk_bytes<Cfg<false, 32, float>>();
template size_t state_bytes<Cfg<true, 64, bf16>>();
template size_t state_bytes<Cfg<false, 32, bf16>>();
template size_t chunk_bytes<Cfg<true, 64, bf16>>();
template size_t chunk_bytes<Cfg<false, 32, bf16>>();

}  // namespace kdn
