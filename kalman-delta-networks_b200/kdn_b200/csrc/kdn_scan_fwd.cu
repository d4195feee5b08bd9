// Forward of the chunked KDN memory scan: one CTA per (value tile, b*h)
// stream walks the chunks in order, keeping its 128 x 64 fp32 slice of the
// state in registers (warp w owns state rows 16w..16w+15).  Per chunk:
//   gated operands -> A, Q (tensor cores) -> T = (I+A)^-1 -> W0 = T Kr, u = T v
//   -> delta = u - W0 (fr*S) -> o = scale (Qr (fr*S) + Q delta)
//   -> S = Diag(2^g_L) S + Diag(fL) Kc^T delta.
// It saves the chunk-start states (bf16) and T, Q (fp32) for the backward.
// Replaces the forward of _chunk_kda_precumsum_paired
// (lit_gpt/kdn_ops/iso_kdn_chunk.py:2037-2086) and of chunk_kalman
// (diag_kdn_chunk.py:3224-3245).
#include "kdn_scan.cuh"

namespace kdn {

template <class CF>
struct FwdLayout {
  static constexpr size_t sz = sizeof(typename CF::OpT);
  static constexpr int C = CF::C;
  // raw inputs of the next chunk land here while the current one finishes
  static constexpr size_t q = 0;
  static constexpr size_t k = q + A128((size_t)C * kKD * 2);
  static constexpr size_t g = k + A128((size_t)C * kKD * 2);
  static constexpr size_t kap = g + A128((size_t)C * kKD * 4);
  static constexpr size_t v = kap + A128(CF::ISO ? (size_t)C * 4 : (size_t)C * kKD * 4);
  static constexpr size_t Kr = v + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t Qr = Kr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Kc = Qr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t As = Kc + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t S = As;  // aliases sA once the solve is done
  static constexpr size_t Del = S + A128((size_t)kKD * CF::LDV * sz);
  static constexpr size_t Qb = As + cmax(A128((size_t)C * CF::LDA * 4), Del - S + A128((size_t)C * CF::LDV * sz));
  static constexpr size_t Tb = Qb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t Ab = Tb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t Xb = Ab + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t W = Xb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t small = W + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t bytes = small + A128(small_floats<CF>() * 4);
};

template <class CF>
__device__ __forceinline__ void bind_fwd_chunk(Chunk<CF>& ch, char* base) {
  using Lo = FwdLayout<CF>;
  using OpT = typename CF::OpT;
  ch.q = reinterpret_cast<bf16*>(base + Lo::q);
  ch.k = reinterpret_cast<bf16*>(base + Lo::k);
  ch.g = reinterpret_cast<float*>(base + Lo::g);
  ch.kap = reinterpret_cast<float*>(base + Lo::kap);
  ch.beta = reinterpret_cast<float*>(base + Lo::kap);
  bind_small(ch, reinterpret_cast<float*>(base + Lo::small));
  ch.Kr = reinterpret_cast<OpT*>(base + Lo::Kr);
  ch.Qr = reinterpret_cast<OpT*>(base + Lo::Qr);
  ch.Kc = reinterpret_cast<OpT*>(base + Lo::Kc);
}

template <class CF>
__global__ void __launch_bounds__(kSeqThreads, 1) scan_fwd_kernel(ScanParams p) {
  using OpT = typename CF::OpT;
  using Lo = FwdLayout<CF>;
  constexpr int C = CF::C;
  constexpr int NTW = C / 16;           // n-tiles per warp job of W0 = T Kr (C x 128)
  constexpr int NJW = kKD / (8 * NTW);  // column jobs per row block
  constexpr int NTU = C / 32;           // n-tiles per warp job of the C x 64 products
  constexpr int NJU = kBV / (8 * NTU);
  static_assert((C / 16) * NJW == 16 && (C / 16) * NJU == 16, "16 warps");
  extern __shared__ __align__(128) char smem[];
  char* base = CF::F32 ? p.dbg + (size_t)(blockIdx.y * gridDim.x + blockIdx.x) * p.dbg_stride : smem;

  Chunk<CF> ch;
  bind_fwd_chunk(ch, base);
  OpT* sTb = reinterpret_cast<OpT*>(base + Lo::Tb);
  OpT* sAb = reinterpret_cast<OpT*>(base + Lo::Ab);
  OpT* sXb = reinterpret_cast<OpT*>(base + Lo::Xb);
  OpT* sW = reinterpret_cast<OpT*>(base + Lo::W);
  OpT* sv = reinterpret_cast<OpT*>(base + Lo::v);
  float* sA = reinterpret_cast<float*>(base + Lo::As);
  OpT* sS = reinterpret_cast<OpT*>(base + Lo::S);
  OpT* sDel = reinterpret_cast<OpT*>(base + Lo::Del);
  OpT* sQb = reinterpret_cast<OpT*>(base + Lo::Qb);

  const int vt = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int warp = threadIdx.x >> 5;
  const int v0 = vt * kBV;
  const bool save_tq = vt == 0 && p.Tsave;

  // state slice: 16 rows x 32 columns per warp
  const int sm0 = 16 * (warp >> 1), sn0 = 32 * (warp & 1);
  float S[1][4][4];
  for_acc<1, 4>(sm0, sn0, [&](int, int nt, int e, int row, int col) {
    S[0][nt][e] = p.S0 ? p.S0[((size_t)bh * kKD + row) * kVD + v0 + col] : 0.f;
  });
  zero_upper_blocks<CF>(sQb);
  zero_upper_blocks<CF>(sTb);

  auto load_qkg = [&](int c) {
    const int t0 = c * C;
    load_raw(ch, p, b, h, t0, min(C, p.T - t0));
  };
  auto load_v = [&](int c) {
    const int t0 = c * C;
    load_tile_op<CF>(sv, CF::LDV, p.v + tok_row(p, b, h, t0) * kVD + v0, (size_t)p.H * kVD, C, min(C, p.T - t0),
                     kBV);
  };
  load_qkg(0);
  load_v(0);
  if constexpr (!CF::F32) cp_async_commit();

  for (int c = 0; c < p.NT; ++c) {
    const int t0 = c * C;
    ch.L = min(C, p.T - t0);
    if constexpr (!CF::F32) cp_async_wait_all();
    __syncthreads();
    prep_chunk(ch);
    __syncthreads();
    const size_t cc = (size_t)bh * p.NT + c;
    chunk_scores(ch, sA, sAb, sQb);
    // the raw inputs are consumed: fetch the next chunk's behind the rest of this one
    if (c + 1 < p.NT) load_qkg(c + 1);
    if constexpr (!CF::F32) cp_async_commit();
    chunk_solve<CF>(sA, sAb, sTb, sXb);
    if (save_tq) {
      store_cc<CF>(static_cast<OpT*>(p.Tsave) + cc * C * C, sTb);
      store_cc<CF>(static_cast<OpT*>(p.Qsave) + cc * C * C, sQb);
    }

    // W0 = T Kr (C x 128), u = T v (C x 64), scaled state operand fr * S
    const int I = warp / NJW;
    {
      float acc[1][NTW][4];
      zero_acc(acc);
      wgemm<1, NTW, true, false>(acc, sTb, CF::LDC, ch.Kr, CF::LDK, 16 * I, (warp % NJW) * 8 * NTW, 0, 16 * (I + 1));
      store_acc(sW, CF::LDK, acc, 16 * I, (warp % NJW) * 8 * NTW);
    }
    const int Iu = warp / NJU, nu = (warp % NJU) * 8 * NTU;
    float u[1][NTU][4];
    zero_acc(u);
    wgemm<1, NTU, true, false>(u, sTb, CF::LDC, sv, CF::LDV, 16 * Iu, nu, 0, 16 * (Iu + 1));
    OpT* hdst = p.h ? static_cast<OpT*>(p.h) + cc * kKD * kVD : nullptr;
    for_acc_pairs<1, 4>(S, sm0, sn0, [&](int, int, int, int row, int col, float x0, float x1) {
      const float f = ch.fr[row];
      st_pair(sS + row * CF::LDV + col, f * x0, f * x1);
      if (hdst) st_pair(hdst + (size_t)row * kVD + v0 + col, x0, x1);
    });
    __syncthreads();
    if (c + 1 < p.NT) load_v(c + 1);
    if constexpr (!CF::F32) cp_async_commit();

    // delta = u - W0 (fr S)
    {
      float acc[1][NTU][4];
      zero_acc(acc);
      wgemm<1, NTU, true, false>(acc, sW, CF::LDK, sS, CF::LDV, 16 * Iu, nu, 0, kKD);
#pragma unroll
      for (int nt = 0; nt < NTU; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[0][nt][e] = u[0][nt][e] - acc[0][nt][e];
      store_acc(sDel, CF::LDV, acc, 16 * Iu, nu);
    }
    __syncthreads();

    // o = scale (Qr (fr S) + Q delta)
    {
      float acc[1][NTU][4];
      zero_acc(acc);
      wgemm<1, NTU, true, false>(acc, ch.Qr, CF::LDK, sS, CF::LDV, 16 * Iu, nu, 0, kKD);
      wgemm<1, NTU, true, false>(acc, sQb, CF::LDC, sDel, CF::LDV, 16 * Iu, nu, 0, 16 * (Iu + 1));
      for_acc_pairs<1, NTU>(acc, 16 * Iu, nu, [&](int, int, int, int row, int col, float x0, float x1) {
        if (row < ch.L) {
          const size_t off = tok_row(p, b, h, t0 + row) * kVD + v0 + col;
          if constexpr (CF::ISO) {
            st_pair(static_cast<bf16*>(p.o) + off, p.scale * x0, p.scale * x1);
          } else {
            st_pair(static_cast<float*>(p.o) + off, p.scale * x0, p.scale * x1);
          }
        }
      });
    }
    // S = Diag(2^g_L) S + Diag(fL) Kc^T delta
    {
      float acc[1][4][4];
      zero_acc(acc);
      wgemm<1, 4, false, false>(acc, ch.Kc, CF::LDK, sDel, CF::LDV, sm0, sn0, 0, C);
      for_acc<1, 4>(sm0, sn0, [&](int, int nt, int e, int row, int) {
        S[0][nt][e] = ch.gL[row] * S[0][nt][e] + ch.fL[row] * acc[0][nt][e];
      });
    }
  }
  if (p.ST) {
    for_acc<1, 4>(sm0, sn0, [&](int, int nt, int e, int row, int col) {
      p.ST[((size_t)bh * kKD + row) * kVD + v0 + col] = S[0][nt][e];
    });
  }
}

template <class CF>
size_t fwd_smem_bytes() {
  return CF::F32 ? 0 : FwdLayout<CF>::bytes;
}
template <class CF>
size_t fwd_dbg_bytes() {
  return CF::F32 ? FwdLayout<CF>::bytes : 0;
}

template <class CF>
int launch_fwd(const ScanParams& p, cudaStream_t st) {
  const size_t smem = fwd_smem_bytes<CF>();
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(scan_fwd_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(scan_fwd_kernel)");
    configured = true;
  }
  dim3 grid(kVD / kBV, p.B * p.H);
  scan_fwd_kernel<CF><<<grid, kSeqThreads, smem, st>>>(p);
  return check_launch("scan_fwd_kernel");
}

template int launch_fwd<Cfg<true, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<true, 64, float>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<false, 32, bf16>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<false, 32, float>>(const ScanParams&, cudaStream_t);
template size_t fwd_dbg_bytes<Cfg<true, 64, float>>();
template size_t fwd_dbg_bytes<Cfg<false, 32, float>>();

}  // namespace kdn
