// Forward of the chunked KDN memory scan, sequential pass: one CTA per
// (value tile, b*h) stream walks the chunks in order, keeping its 128 x 64
// fp32 slice of the state in registers (warp w < 16 owns rows 16(w/2)..,
// columns 32(w%2)..).  A 17th, producer warp streams the chunk records of
// scan_prep_kernel and the value rows into a ring of NS shared-memory stages
// with bulk copies (full / empty mbarriers, bounded waits); the 16 compute
// warps synchronise among themselves with a named barrier.  Per chunk:
//   S' = fr * S (bf16, also the saved chunk-start state h)
//   delta = T v - W0 S'
//   o = scale (Qr S' + Q delta)
//   S = Diag(2^g_L) S + Diag(fL) Kc^T delta
// Replaces the inter-chunk half of _chunk_kda_fwd_precum
// (lit_gpt/kdn_ops/iso_kdn_chunk.py:2037-2086: chunk_gated_delta_rule_fwd_h
// and the output stage) and of _diag_kdn_memory_forward
// (diag_kdn_chunk.py:3224-3245).
#include "kdn_scan.cuh"

namespace kdn {

template <class CF>
struct FwdLayout {
  static constexpr size_t sz = sizeof(typename CF::OpT);
  static constexpr int C = CF::C;
  static constexpr int NS = CF::F32 ? 1 : (CF::ISO ? 2 : 4);
  // stage: the chunk record, then the value rows [C][LDV]
  static constexpr size_t v = Rec<CF>::bytes;
  static constexpr size_t stage = A128(v + (size_t)C * CF::LDV * sz);
  static constexpr size_t S = NS * stage;  // two [KD][LDV] buffers
  static constexpr size_t Del = S + 2 * state_block_bytes<CF>();
  static constexpr size_t bar = Del + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t bytes = bar + 128;  // full[NS], empty[NS]
};

template <class CF>
__global__ void __launch_bounds__(kSeqThreads + 32, 1) scan_fwd_kernel(ScanParams p) {
  using OpT = typename CF::OpT;
  using Lo = FwdLayout<CF>;
  using R = Rec<CF>;
  constexpr int C = CF::C, NS = Lo::NS;
  constexpr int NTU = C / 32;  // n-tiles per warp job of the C x 64 products
  constexpr int NJU = kBV / (8 * NTU);
  static_assert((C / 16) * NJU == 16, "16 warps");
  extern __shared__ __align__(128) char smem[];
  char* base = CF::F32 ? p.dbg + (size_t)(blockIdx.y * gridDim.x + blockIdx.x) * p.dbg_stride : smem;

  const int vt = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int v0 = vt * kBV;
  const char* recs = static_cast<const char*>(p.rec) + (size_t)bh * p.NT * R::bytes;
  char* hout = static_cast<char*>(p.h) + ((size_t)bh * p.NT * (kVD / kBV) + vt) * state_block_bytes<CF>();
  constexpr size_t h_stride = (kVD / kBV) * state_block_bytes<CF>();  // per chunk
  uint64_t* full = reinterpret_cast<uint64_t*>(base + Lo::bar);
  uint64_t* empty = full + NS;
  OpT* sDel = reinterpret_cast<OpT*>(base + Lo::Del);

  // chunk c's record and value rows into stage c % NS (producer warp)
  auto issue = [&](int c) {
    char* st = base + (c % NS) * Lo::stage;
    const int t0 = c * C, L = min(C, p.T - t0);
    if (lane == 0) {
      mbar_expect_tx(&full[c % NS], (unsigned)(R::bytes + (size_t)L * kBV * 2));
      bulk_g2s(st, recs + (size_t)c * R::bytes, (unsigned)R::bytes, &full[c % NS]);
    }
    __syncwarp();
    for (int r = lane; r < L; r += 32)
      bulk_g2s(st + Lo::v + (size_t)r * CF::LDV * sizeof(OpT), p.v + tok_row(p, b, h, t0 + r) * kVD + v0, kBV * 2,
               &full[c % NS]);
  };
  // fp32 debug precision: synchronous copies by the whole block
  auto load_sync = [&](int c) {
    const int t0 = c * C, L = min(C, p.T - t0);
    copy_block<CF>(base, recs + (size_t)c * R::bytes, R::bytes);
    load_tile_op<CF>(reinterpret_cast<OpT*>(base + Lo::v), CF::LDV, p.v + tok_row(p, b, h, t0) * kVD + v0,
                     (size_t)p.H * kVD, C, L, kBV);
  };

  if constexpr (!CF::F32) {
    if (threadIdx.x == 0) {
      for (int s = 0; s < NS; ++s) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], kSeqThreads / 32);
      }
      fence_mbar_init();
    }
    __syncthreads();
    // producer warp: refill a stage once all 16 compute warps released it
    if (warp == kSeqThreads / 32) {
      for (int c = 0; c < p.NT; ++c) {
        if (c >= NS) mbar_wait(&empty[c % NS], (c / NS - 1) & 1, p.status);
        issue(c);
      }
      return;
    }
  }

  const int sm0 = 16 * (warp >> 1), sn0 = 32 * (warp & 1);
  float S[1][4][4];
  for_acc<1, 4>(sm0, sn0, [&](int, int nt, int e, int row, int col) {
    S[0][nt][e] = p.S0 ? p.S0[((size_t)bh * kKD + row) * kVD + v0 + col] : 0.f;
  });
  const int Iu = warp / NJU, nu = (warp % NJU) * 8 * NTU;

  for (int c = 0; c < p.NT; ++c) {
    const int t0 = c * C, L = min(C, p.T - t0);
    char* st = base + (c % NS) * Lo::stage;
    const OpT* sQr = reinterpret_cast<const OpT*>(st + R::Qr);
    const OpT* sKc = reinterpret_cast<const OpT*>(st + R::Kc);
    const OpT* sW0 = reinterpret_cast<const OpT*>(st + R::W0);
    const OpT* sT = reinterpret_cast<const OpT*>(st + R::T);
    const OpT* sQ = reinterpret_cast<const OpT*>(st + R::Q);
    const float* fr = reinterpret_cast<const float*>(st + R::F);
    const float* fL = fr + kKD;
    const float* gL = fL + kKD;
    OpT* sv = reinterpret_cast<OpT*>(st + Lo::v);
    OpT* sS = reinterpret_cast<OpT*>(base + Lo::S + (c & 1) * state_block_bytes<CF>());

    if constexpr (CF::F32) {
      __syncthreads();
      load_sync(c);
      __syncthreads();
    } else {
      mbar_wait(&full[c % NS], (c / NS) & 1, p.status);
      for (int e = threadIdx.x; e < (C - L) * (kBV / 8); e += kSeqThreads)
        *reinterpret_cast<int4*>(sv + (L + e / (kBV / 8)) * CF::LDV + (e % (kBV / 8)) * 8) = make_int4(0, 0, 0, 0);
    }
    // S' = fr S: the product operand and the saved chunk-start state
    for_acc_pairs<1, 4>(S, sm0, sn0, [&](int, int, int, int row, int col, float x0, float x1) {
      const float f = fr[row];
      st_pair(sS + row * CF::LDV + col, f * x0, f * x1);
    });
    if constexpr (!CF::F32) fence_async_shared();
    bar_sync(1, kSeqThreads);
    if constexpr (CF::F32) {
      copy_block<CF>(hout + c * h_stride, sS, state_block_bytes<CF>());
    } else {
      if (threadIdx.x == 32) {
        bulk_s2g(hout + c * h_stride, sS, (unsigned)state_block_bytes<CF>());
        bulk_commit();
      }
    }

    // delta = T v - W0 S'
    {
      float u[1][NTU][4], a[1][NTU][4];
      zero_acc(u);
      zero_acc(a);
      wgemm<1, NTU, true, false>(u, sT, CF::LDC, sv, CF::LDV, 16 * Iu, nu, 0, 16 * (Iu + 1));
      wgemm<1, NTU, true, false>(a, sW0, CF::LDK, sS, CF::LDV, 16 * Iu, nu, 0, kKD);
#pragma unroll
      for (int nt = 0; nt < NTU; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) u[0][nt][e] -= a[0][nt][e];
      store_acc(sDel, CF::LDV, u, 16 * Iu, nu);
    }
    // the h store of chunk c - 1 has read its buffer (rewritten by chunk c + 1)
    if constexpr (!CF::F32)
      if (threadIdx.x == 32) bulk_wait_read<1>();
    bar_sync(1, kSeqThreads);

    // o = scale (Qr S' + Q delta)
    {
      float acc[1][NTU][4];
      zero_acc(acc);
      wgemm<1, NTU, true, false>(acc, sQr, CF::LDK, sS, CF::LDV, 16 * Iu, nu, 0, kKD);
      wgemm<1, NTU, true, false>(acc, sQ, CF::LDC, sDel, CF::LDV, 16 * Iu, nu, 0, 16 * (Iu + 1));
      for_acc_pairs<1, NTU>(acc, 16 * Iu, nu, [&](int, int, int, int row, int col, float x0, float x1) {
        if (row < L) {
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
      wgemm<1, 4, false, false>(acc, sKc, CF::LDK, sDel, CF::LDV, sm0, sn0, 0, C);
      for_acc<1, 4>(sm0, sn0, [&](int, int nt, int e, int row, int) {
        S[0][nt][e] = gL[row] * S[0][nt][e] + fL[row] * acc[0][nt][e];
      });
    }
    if constexpr (!CF::F32) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[c % NS]);  // this warp is done with the stage
    }
  }
  if (p.ST) {
    for_acc<1, 4>(sm0, sn0, [&](int, int nt, int e, int row, int col) {
      p.ST[((size_t)bh * kKD + row) * kVD + v0 + col] = S[0][nt][e];
    });
  }
  if constexpr (!CF::F32)
    if (threadIdx.x == 32) bulk_wait_all();
}

template <class CF>
size_t fwd_dbg_bytes() {
  return CF::F32 ? FwdLayout<CF>::bytes : 0;
}

template <class CF> int launch_prep(const ScanParams&, cudaStream_t);

template <class CF>
int launch_fwd(const ScanParams& p, cudaStream_t st) {
  int rc = launch_prep<CF>(p, st);
  if (rc != KDN_OK) return rc;
  const size_t smem = CF::F32 ? 0 : FwdLayout<CF>::bytes;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(scan_fwd_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(scan_fwd_kernel)");
    configured = true;
  }
  dim3 grid(kVD / kBV, p.B * p.H);
  scan_fwd_kernel<CF><<<grid, CF::F32 ? kSeqThreads : kSeqThreads + 32, smem, st>>>(p);
  return check_launch("scan_fwd_kernel");
}

template int launch_fwd<Cfg<true, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<true, 64, float>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<false, 32, bf16>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<false, 32, float>>(const ScanParams&, cudaStream_t);
template size_t fwd_dbg_bytes<Cfg<true, 64, float>>();
template size_t fwd_dbg_bytes<Cfg<false, 32, float>>();

}  // namespace kdn
