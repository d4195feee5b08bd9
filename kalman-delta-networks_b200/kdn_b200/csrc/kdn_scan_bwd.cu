// Backward of the chunked KDN memory scan.
//
// 1. scan_bwd_state_kernel (one CTA per (value tile, b*h), chunks in reverse):
//    carries the state adjoint dS in registers; a producer warp streams the
//    chunk records of the forward's first pass and the dO rows through a
//    ring of bulk-copy stages,
//        ddelta  = scale Q^T dO + Kc (fL*dS)
//        dS_prev = Diag(2^g_L) dS + Diag(fr) (scale Qr^T dO - W0^T ddelta)
//    and stores every chunk's fL-scaled chunk-end adjoint (bf16) for step 2.
// 2. scan_bwd_chunk_kernel (one CTA per (chunk, b*h), all chunks in parallel):
//    with the saved chunk-start state S0' = fr S0 and chunk-end adjoint
//    dS'' = fL dS it
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
#include "kdn_tc.cuh"
#include "kdn_tma.cuh"

namespace kdn {

// ---------------------------------------------------------------------------
// 1. reverse state-adjoint sweep
// ---------------------------------------------------------------------------
// Stage: the chunk record, then dO [C][LDV] OpT (iso) or fp32 [C][BV]
// staging (diag, rounded to bf16 into the dOb buffer).
template <class CF>
struct StateLayout {
  static constexpr size_t sz = sizeof(typename CF::OpT);
  static constexpr int C = CF::C;
  static constexpr int NS = CF::F32 ? 1 : (CF::ISO ? 2 : 4);
  static constexpr bool STAGE_F32 = !CF::ISO;  // diag cotangent arrives as fp32
  static constexpr size_t dO = Rec<CF>::bytes;
  static constexpr size_t stage = A128(dO + (STAGE_F32 ? (size_t)C * kBV * 4 : (size_t)C * CF::LDV * sz));
  static constexpr size_t dOb = NS * stage;  // diag: the rounded operand
  static constexpr size_t DS = dOb + A128(STAGE_F32 ? (size_t)C * CF::LDV * sz : 16);  // two [KD][LDV] buffers
  static constexpr size_t DD = DS + 2 * state_block_bytes<CF>();
  static constexpr size_t bar = DD + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t bytes = bar + 128;
};

template <class CF>
__global__ void __launch_bounds__(kSeqThreads + 32, 1) scan_bwd_state_kernel(ScanParams p) {
  using OpT = typename CF::OpT;
  using Lo = StateLayout<CF>;
  using R = Rec<CF>;
  constexpr int C = CF::C, NS = Lo::NS;
  constexpr int NTU = C / 32;
  constexpr int NJU = kBV / (8 * NTU);
  static_assert((C / 16) * NJU == 16, "16 warps");
  extern __shared__ __align__(128) char smem[];
  char* base = CF::F32 ? p.dbg + (size_t)(blockIdx.y * gridDim.x + blockIdx.x) * p.dbg_stride : smem;

  const int vt = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int v0 = vt * kBV;
  const char* recs = static_cast<const char*>(p.rec) + (size_t)bh * p.NT * R::bytes;
  char* dhout = static_cast<char*>(p.dh) + ((size_t)bh * p.NT * (kVD / kBV) + vt) * state_block_bytes<CF>();
  constexpr size_t h_stride = (kVD / kBV) * state_block_bytes<CF>();
  uint64_t* full = reinterpret_cast<uint64_t*>(base + Lo::bar);
  uint64_t* empty = full + NS;
  OpT* sDD = reinterpret_cast<OpT*>(base + Lo::DD);
  constexpr unsigned dO_row = Lo::STAGE_F32 ? kBV * 4 : kBV * 2;
  constexpr size_t dO_pitch = Lo::STAGE_F32 ? (size_t)kBV * 4 : (size_t)CF::LDV * Lo::sz;

  // the it-th chunk from the end into stage it % NS (producer warp)
  auto issue = [&](int it) {
    const int c = p.NT - 1 - it;
    char* st = base + (it % NS) * Lo::stage;
    const int t0 = c * C, L = min(C, p.T - t0);
    if (lane == 0) {
      mbar_expect_tx(&full[it % NS], (unsigned)(R::bytes + (size_t)L * dO_row));
      bulk_g2s(st, recs + (size_t)c * R::bytes, (unsigned)R::bytes, &full[it % NS]);
    }
    __syncwarp();
    const char* src = static_cast<const char*>(p.dO) + (Lo::STAGE_F32 ? 4 : 2) * (size_t)v0;
    const size_t row_bytes = (Lo::STAGE_F32 ? 4 : 2) * (size_t)kVD;
    for (int r = lane; r < L; r += 32)
      bulk_g2s(st + Lo::dO + r * dO_pitch, src + tok_row(p, b, h, t0 + r) * row_bytes, dO_row, &full[it % NS]);
  };
  auto load_sync = [&](int it) {
    const int c = p.NT - 1 - it;
    const int t0 = c * C, L = min(C, p.T - t0);
    copy_block<CF>(base, recs + (size_t)c * R::bytes, R::bytes);
    const size_t r0 = tok_row(p, b, h, t0) * kVD + v0;
    if constexpr (CF::ISO) {
      load_tile_op<CF>(reinterpret_cast<OpT*>(base + Lo::dO), CF::LDV, static_cast<const bf16*>(p.dO) + r0,
                       (size_t)p.H * kVD, C, L, kBV);
    } else {
      copy_rows<false>(base + Lo::dO, kBV * 4, static_cast<const float*>(p.dO) + r0, (size_t)p.H * kVD * 4, C, L,
                       kBV * 4);
    }
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
    if (warp == kSeqThreads / 32) {
      for (int it = 0; it < p.NT; ++it) {
        if (it >= NS) mbar_wait(&empty[it % NS], (it / NS - 1) & 1, p.status);
        issue(it);
      }
      return;
    }
  }

  const int sm0 = 16 * (warp >> 1), sn0 = 32 * (warp & 1);
  float dS[1][4][4];
  for_acc<1, 4>(sm0, sn0, [&](int, int nt, int e, int row, int col) {
    dS[0][nt][e] = p.dST ? p.dST[((size_t)bh * kKD + row) * kVD + v0 + col] : 0.f;
  });
  const int Iu = warp / NJU, nu = (warp % NJU) * 8 * NTU;

  for (int it = 0; it < p.NT; ++it) {
    const int c = p.NT - 1 - it;
    const int L = min(C, p.T - c * C);
    char* st = base + (it % NS) * Lo::stage;
    const OpT* sQr = reinterpret_cast<const OpT*>(st + R::Qr);
    const OpT* sKc = reinterpret_cast<const OpT*>(st + R::Kc);
    const OpT* sW0 = reinterpret_cast<const OpT*>(st + R::W0);
    const OpT* sQ = reinterpret_cast<const OpT*>(st + R::Q);
    const float* fr = reinterpret_cast<const float*>(st + R::F);
    const float* fL = fr + kKD;
    const float* gL = fL + kKD;
    OpT* sdO = reinterpret_cast<OpT*>(Lo::STAGE_F32 ? base + Lo::dOb : st + Lo::dO);
    OpT* sDS = reinterpret_cast<OpT*>(base + Lo::DS + (it & 1) * state_block_bytes<CF>());

    if constexpr (CF::F32) {
      __syncthreads();
      load_sync(it);
      __syncthreads();
    } else {
      mbar_wait(&full[it % NS], (it / NS) & 1, p.status);
      if constexpr (CF::ISO) {
        for (int e = threadIdx.x; e < (C - L) * (kBV / 8); e += kSeqThreads)
          *reinterpret_cast<int4*>(sdO + (L + e / (kBV / 8)) * CF::LDV + (e % (kBV / 8)) * 8) =
              make_int4(0, 0, 0, 0);
      }
    }
    if constexpr (Lo::STAGE_F32) {
      // the reference rounds the fp32 cotangent to bf16 first (diag_kdn_chunk.py:3277)
      const float* stg = reinterpret_cast<const float*>(st + Lo::dO);
      for (int e = threadIdx.x; e < C * kBV / 2; e += kSeqThreads) {
        const int i = (2 * e) / kBV, cc = 2 * e - i * kBV;
        float2 x = make_float2(0.f, 0.f);
        if (i < L) x = *reinterpret_cast<const float2*>(stg + i * kBV + cc);
        st_pair(sdO + i * CF::LDV + cc, __bfloat162float(__float2bfloat16_rn(x.x)),
                __bfloat162float(__float2bfloat16_rn(x.y)));
      }
    }
    // dS'' = fL dS: the product operand and the saved chunk-end adjoint
    for_acc_pairs<1, 4>(dS, sm0, sn0, [&](int, int, int, int row, int col, float x0, float x1) {
      const float f = fL[row];
      st_pair(sDS + row * CF::LDV + col, f * x0, f * x1);
    });
    if constexpr (!CF::F32) fence_async_shared();
    bar_sync(1, kSeqThreads);
    if constexpr (CF::F32) {
      copy_block<CF>(dhout + c * h_stride, sDS, state_block_bytes<CF>());
    } else {
      if (threadIdx.x == 32) {
        bulk_s2g(dhout + c * h_stride, sDS, (unsigned)state_block_bytes<CF>());
        bulk_commit();
      }
    }

    // Qr^T dO (independent of the carried adjoint)
    float a1[1][4][4];
    zero_acc(a1);
    wgemm<1, 4, false, false>(a1, sQr, CF::LDK, sdO, CF::LDV, sm0, sn0, 0, C);
    // ddelta = scale Q^T dO + Kc dS''
    {
      float u[1][NTU][4], a[1][NTU][4];
      zero_acc(u);
      zero_acc(a);
      wgemm<1, NTU, false, false>(u, sQ, CF::LDC, sdO, CF::LDV, 16 * Iu, nu, 16 * Iu, C);
      wgemm<1, NTU, true, false>(a, sKc, CF::LDK, sDS, CF::LDV, 16 * Iu, nu, 0, kKD);
#pragma unroll
      for (int nt = 0; nt < NTU; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) u[0][nt][e] = p.scale * u[0][nt][e] + a[0][nt][e];
      store_acc(sDD, CF::LDV, u, 16 * Iu, nu);
    }
    if constexpr (!CF::F32)
      if (threadIdx.x == 32) bulk_wait_read<1>();
    bar_sync(1, kSeqThreads);

    // dS <- Diag(2^g_L) dS + Diag(fr) (scale Qr^T dO - W0^T ddelta)
    {
      float a2[1][4][4];
      zero_acc(a2);
      wgemm<1, 4, false, false>(a2, sW0, CF::LDK, sDD, CF::LDV, sm0, sn0, 0, C);
      for_acc<1, 4>(sm0, sn0, [&](int, int nt, int e, int row, int) {
        dS[0][nt][e] = gL[row] * dS[0][nt][e] + fr[row] * (p.scale * a1[0][nt][e] - a2[0][nt][e]);
      });
    }
    if constexpr (!CF::F32) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[it % NS]);
    }
  }
  if (p.dS0) {
    for_acc<1, 4>(sm0, sn0, [&](int, int nt, int e, int row, int col) {
      p.dS0[((size_t)bh * kKD + row) * kVD + v0 + col] = dS[0][nt][e];
    });
  }
  if constexpr (!CF::F32)
    if (threadIdx.x == 32) bulk_wait_all();
}

// Tensor-core reverse sweep (bf16 precision): two CTAs per (b, h) stream, each
// with 64 value columns of the 128 x 128 fp32 adjoint in TMEM; same roles as
// the tensor-core forward (8 data warps, one MMA thread, one producer warp).  Per chunk, with the
// record's folded factors (Qs = scale fr Qr, Kf = fL Kc, Wf = fr W0,
// Qq = scale Q):
//   dS -> bf16 operand (saved as dh);  dS <- 2^g_L dS           (TMEM ld / st)
//   ddelta^T = dO^T Qq + dS^T Kf^T, Qq read as its transpose Qt (MMA, M = 64 values)
//   dS += Qs^T dO - Wf^T ddelta                                  (MMA, M = 128 keys)
template <class CF>
struct StateTcLayout {
  static constexpr int C = CF::C;
  static constexpr int NS = CF::C == 64 ? 2 : 3;
  static constexpr bool DF32 = !CF::ISO;  // the diagonal variant's cotangent arrives as fp32 rows
  using R = RecTc<CF>;
  static constexpr size_t rec = R::bytes - R::bwd_begin;  // the record from Qs on
  static constexpr size_t dO = rec;  // iso: [C][64] bf16 swizzled; diag: [C][64] fp32
  static constexpr size_t stage = align_up(dO + (size_t)C * (DF32 ? 256 : 128), 1024);
  static constexpr size_t dOb = NS * stage;  // diag: the bf16-rounded operand [C][64]
  static constexpr size_t DS = dOb + (DF32 ? align_up((size_t)C * 128, 1024) : 0);  // [KD][64] (also dh)
  static constexpr size_t DD = DS + (size_t)kKD * 128;                               // ddelta^T [64][C]
  static constexpr size_t bar = DD + align_up((size_t)C * 128, 1024);
  static constexpr size_t bytes = bar + 128 + 1024;
};

template <class CF>
__global__ void __launch_bounds__(kTcThreads, 1) scan_bwd_state_tc_kernel(ScanParams p,
                                                                          const __grid_constant__ TcMaps maps) {
  using Lo = StateTcLayout<CF>;
  using R = RecTc<CF>;
  constexpr int C = CF::C, NS = Lo::NS, HC = C / 2;
  constexpr uint32_t TS = 0, TD = 64;  // TMEM columns: adjoint, ddelta^T
  constexpr int NTH = kTcWarps * 32;
  extern __shared__ __align__(1024) char smem_raw[];
  char* base = align1024(smem_raw);

  const SeqStream ss = seq_stream(p, blockIdx.x);
  const int vh = blockIdx.y, V0 = 64 * vh, b = ss.b, h = ss.h, c_lo = ss.c_lo, c_hi = ss.c_hi;
  const bool vl = p.vl.on();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const char* recs = static_cast<const char*>(p.rec) + ss.rec_row * p.NT * R::bytes;
  char* dhout =
      static_cast<char*>(p.dh) + ss.rec_row * p.NT * 2 * hblock_bytes<CF>() + (size_t)vh * hblock_bytes<CF>();
  uint64_t* full = reinterpret_cast<uint64_t*>(base + Lo::bar);
  uint64_t* empty = full + NS;
  uint64_t* mmab = empty + NS;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mmab + 1);
  char* sDS = base + Lo::DS;
  char* sDD = base + Lo::DD;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(mmab, 1);
    fence_mbar_init();
  }
  if (warp == 0) tc::alloc(tslot, 256);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tslot;

  if (warp == kTcWarps) {
    for (int it = 0; it < c_hi - c_lo; ++it) {
      const int s = it % NS, c = c_hi - 1 - it;
      if (it >= NS) mbar_wait(&empty[s], (it / NS - 1) & 1, p.status);
      if (lane == 0) {
        char* st = base + s * Lo::stage;
        int t0, L;
        chunk_span<C>(p, c, t0, L);
        mbar_expect_tx(&full[s], (unsigned)(Lo::rec + (size_t)C * (Lo::DF32 ? 256 : 128)));
        bulk_g2s(st, recs + (size_t)c * R::bytes + R::bwd_begin, (unsigned)Lo::rec, &full[s]);
        tma_load_4d(st + Lo::dO, &maps.in, V0, h, t0, b, &full[s]);
      }
      __syncwarp();
    }
    return;
  }

  const int q = warp & 3, hf = warp >> 2;
  const int row = 32 * q + lane;  // key (adjoint)
  const int vc = 16 * q + lane;   // value column of this CTA (ddelta^T, M = 64: lanes < 16)
  const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
  for (int j = 0; j < 32; j += 16) {
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = p.dST ? p.dST[(ss.state * kKD + row) * kVD + V0 + 32 * hf + j + i] : 0.f;
    tc::st16(tl + TS + 32 * hf + j, x);
  }
  tc::wait_st();
  uint32_t mph = 0;

  for (int it = 0; it < c_hi - c_lo; ++it) {
    const int s = it % NS, c = c_hi - 1 - it;
    char* st = base + s * Lo::stage;
    char* sdO = Lo::DF32 ? base + Lo::dOb : st + Lo::dO;
    // rows past a packed sequence's end (its last chunk's box ran into the
    // next sequence) are zeroed
    int L = C;
    if (vl) {
      int t0;
      chunk_span<C>(p, c, t0, L);
    }
    mbar_wait(&full[s], (it / NS) & 1, p.status);
    if constexpr (Lo::DF32) {
      // the reference rounds the fp32 cotangent to bf16 first (diag_kdn_chunk.py:3277)
      const float* src = reinterpret_cast<const float*>(st + Lo::dO);
      for (int e = threadIdx.x; e < C * 8; e += NTH) {
        const int r = e >> 3, g = e & 7;
        float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (r < L) ld8(x, src + r * 64 + 8 * g);
        st8(reinterpret_cast<bf16*>(sdO + tc::sw_off(r, 8 * g, C)), x);
      }
    } else {
      if (L < C) zero_tail_rows<C>(sdO, L, threadIdx.x, NTH);
    }
    {
      // adjoint operand (and dh), then dS <- 2^g_L dS
      const float gl = reinterpret_cast<const float*>(st + (R::F - R::bwd_begin))[2 * kKD + row];
#pragma unroll
      for (int j = 0; j < 32; j += 16) {
        float x[16];
        tc::ld16(tl + TS + 32 * hf + j, x);
        tc::st_row16(sDS, kKD, row, 32 * hf + j, x, 1.f);
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] *= gl;
        tc::st16(tl + TS + 32 * hf + j, x);
      }
      // the scaled adjoint's TMEM stores complete before the adjoint MMAs (wait_st below)
    }
    fence_async_shared();
    tc::fence_before();
    bar_sync(1, NTH);
    if (threadIdx.x == 32) {
      bulk_s2g(dhout + (size_t)c * 2 * hblock_bytes<CF>(), sDS, (unsigned)hblock_bytes<CF>());
      bulk_commit();
    }
    if (threadIdx.x == 0) {
      tc::fence_after();
      constexpr uint32_t id2 = tc::idesc(64, C, true, false);
      for (int ks = 0; ks < C / 16; ++ks)
        tc::mma(tmem + TD, tc::desc_mn(sdO, C, ks), tc::desc_k(st + (R::Qt - R::bwd_begin), C, ks), id2, ks > 0);
      for (int ks = 0; ks < kKD / 16; ++ks)
        tc::mma(tmem + TD, tc::desc_mn(sDS, kKD, ks), tc::desc_k(st + (R::Kf - R::bwd_begin), C, ks), id2, true);
      tc::commit(mmab);
    }
    mbar_wait(mmab, mph, p.status);
    mph ^= 1;
    tc::fence_after();
    // ddelta^T (value row vc, lanes < 16) -> bf16 operand tile [64][C]
#pragma unroll
    for (int j = 0; j < HC; j += 16) {
      float x[16];
      tc::ld16(tl + TD + HC * hf + j, x);
      if (lane < 16) tc::st_row16(sDD, 64, vc, HC * hf + j, x, 1.f);
    }
    if (threadIdx.x == 32) bulk_wait_read<0>();  // dh has left the adjoint operand (rewritten next chunk)
    tc::wait_st();
    fence_async_shared();
    tc::fence_before();
    bar_sync(1, NTH);
    if (threadIdx.x == 0) {
      tc::fence_after();
      constexpr uint32_t ids = tc::idesc(128, 64, true, true), idn = tc::idesc(128, 64, true, false, true);
      for (int ks = 0; ks < C / 16; ++ks)
        tc::mma(tmem + TS, tc::desc_mn(st + (R::Qs - R::bwd_begin), C, ks), tc::desc_mn(sdO, C, ks), ids, true);
      for (int ks = 0; ks < C / 16; ++ks)
        tc::mma(tmem + TS, tc::desc_mn(st + (R::Wf - R::bwd_begin), C, ks), tc::desc_k(sDD, 64, ks), idn, true);
      tc::commit(&empty[s]);
      tc::commit(mmab);
    }
    mbar_wait(mmab, mph, p.status);
    mph ^= 1;
    tc::fence_after();
  }
  if (p.dS0) {
    for (int j = 0; j < 32; j += 16) {
      float x[16];
      tc::ld16(tl + TS + 32 * hf + j, x);
#pragma unroll
      for (int i = 0; i < 16; ++i) p.dS0[(ss.state * kKD + row) * kVD + V0 + 32 * hf + j + i] = x[i];
    }
  }
  if (threadIdx.x == 32) bulk_wait_all();
  tc::fence_before();
  bar_sync(1, NTH);
  if (warp == 0) {
    tc::fence_after();
    tc::dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------------------
// 2. chunk-parallel gradients
// ---------------------------------------------------------------------------
// The diagonal variant's fp32 cotangent as the OpT operand, rounded to bf16
// like the reference does before its backward kernels (diag_kdn_chunk.py:3277).
template <class CF>
__device__ __forceinline__ void convert_dO(typename CF::OpT* dst, const float* st) {
  for (int e = threadIdx.x; e < CF::C * kBV / 2; e += blockDim.x) {
    const int i = (2 * e) / kBV, c = 2 * e - i * kBV;
    const float2 x = *reinterpret_cast<const float2*>(st + i * kBV + c);
    const float a = __bfloat162float(__float2bfloat16_rn(x.x)), b = __bfloat162float(__float2bfloat16_rn(x.y));
    st_pair(dst + i * CF::LDV + c, a, b);
  }
}

template <class CF>
struct ChunkLayout {
  static constexpr size_t sz = sizeof(typename CF::OpT);
  static constexpr int C = CF::C;
  static constexpr int LDO = kKD + 8;  // fp32 gradient pitch: conflict-free pair stores
  // raw inputs (fetched a second time after the value loop, for the gate mapping)
  static constexpr size_t q = 0;
  static constexpr size_t k = q + A128((size_t)C * kKD * 2);
  static constexpr size_t g = k + A128((size_t)C * kKD * 2);
  static constexpr size_t kap = g + A128((size_t)C * kKD * 4);
  static constexpr size_t raw_end = kap + A128(CF::ISO ? (size_t)C * 4 : (size_t)C * kKD * 4);
  // one value half: v, dO [C][LDV]; S0', dS'' [KD][LDV]; diag fp32 dO staging
  static constexpr size_t hv = 0;
  static constexpr size_t hdO = hv + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t hS0 = hdO + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t hdS = hS0 + state_block_bytes<CF>();
  static constexpr size_t hdOst = hdS + state_block_bytes<CF>();
  static constexpr size_t half_bytes = hdOst + A128(CF::ISO ? 16 : (size_t)C * kBV * 4);
  // region 1: the raw inputs, or the second value half next to delta and ddelta
  static constexpr size_t setA = 0;
  static constexpr size_t Del = setA + half_bytes;
  static constexpr size_t DD = Del + A128((size_t)C * CF::LDV * sz);
  static constexpr size_t r1_end = cmax(raw_end, DD + A128((size_t)C * CF::LDV * sz));
  // region 2: the first value half, or after the loop the post-loop buffers
  // (dA and dQ first: the exact path of the gate mapping still reads them)
  static constexpr size_t setB = r1_end;
  static constexpr size_t dA = r1_end;
  static constexpr size_t dQ = dA + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t dW = dQ + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t dT = dW + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t X = dT + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t r2_end = cmax(setB + half_bytes, X + A128((size_t)C * CF::LDC * sz));
  static constexpr size_t Kr = r2_end;
  static constexpr size_t Qr = Kr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Kc = Qr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Tb = Kc + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Qb = Tb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t W = Qb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t small = W + A128((size_t)C * CF::LDK * sz);
  // small: chunk scalars, cfl[KD], cgl[KD]
  static constexpr size_t bytes = small + A128((small_floats<CF>() + 2 * kKD) * 4);
  // fp32 gradient operands of the gate mapping (over dW .. W, dead by then)
  static constexpr size_t xk = dW;  // dKr [C][LDO]
  static constexpr size_t xq = xk + A128((size_t)C * LDO * 4);
  static constexpr size_t xc = xq + A128((size_t)C * LDO * 4);
  static constexpr size_t x_end = xc + A128((size_t)C * LDO * 4);
  static_assert(x_end <= small, "gradient operands fit in the dead operand buffers");
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
  bf16* rq_ = reinterpret_cast<bf16*>(base + Lo::q);
  bf16* rk_ = reinterpret_cast<bf16*>(base + Lo::k);
  float* rg_ = reinterpret_cast<float*>(base + Lo::g);
  float* rkap_ = reinterpret_cast<float*>(base + Lo::kap);
  ch.Kr = reinterpret_cast<OpT*>(base + Lo::Kr);
  ch.Qr = reinterpret_cast<OpT*>(base + Lo::Qr);
  ch.Kc = reinterpret_cast<OpT*>(base + Lo::Kc);
  float* small = reinterpret_cast<float*>(base + Lo::small);
  bind_small(ch, small);
  float* cfl = small + small_floats<CF>();
  float* cgl = cfl + kKD;
  OpT* sDel = reinterpret_cast<OpT*>(base + Lo::Del);
  OpT* sDD = reinterpret_cast<OpT*>(base + Lo::DD);
  OpT* sdW = reinterpret_cast<OpT*>(base + Lo::dW);
  OpT* sdT = reinterpret_cast<OpT*>(base + Lo::dT);
  OpT* sX = reinterpret_cast<OpT*>(base + Lo::X);
  OpT* sdA = reinterpret_cast<OpT*>(base + Lo::dA);
  OpT* sdQ = reinterpret_cast<OpT*>(base + Lo::dQ);
  OpT* sTb = reinterpret_cast<OpT*>(base + Lo::Tb);
  OpT* sQb = reinterpret_cast<OpT*>(base + Lo::Qb);
  OpT* sW = reinterpret_cast<OpT*>(base + Lo::W);

  const int c = p.c_lo + blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = c * C;
  const int L = min(C, p.T - t0);
  const size_t cc = (size_t)bh * p.NT + c;
  ch.L = L;

  const char* hsrc = static_cast<const char*>(p.h) + cc * (kVD / kBV) * hblock_bytes<CF>();
  const char* dhsrc = static_cast<const char*>(p.dh) + cc * (kVD / kBV) * hblock_bytes<CF>();
  // value half vh: the first in region 2, the second over the consumed raw inputs
  auto half_base = [&](int vh) { return base + (vh == 0 ? Lo::setB : Lo::setA); };
  auto issue_half = [&](int vh) {
    char* hb = half_base(vh);
    const int v0 = vh * kBV;
    const size_t r0 = tok_row(p, b, h, t0);
    load_tile_op<CF>(reinterpret_cast<OpT*>(hb + Lo::hv), CF::LDV, p.v + r0 * kVD + v0, (size_t)p.H * kVD, C, L,
                     kBV);
    if constexpr (CF::ISO) {
      load_tile_op<CF>(reinterpret_cast<OpT*>(hb + Lo::hdO), CF::LDV, static_cast<const bf16*>(p.dO) + r0 * kVD + v0,
                       (size_t)p.H * kVD, C, L, kBV);
    } else {
      copy_rows<!CF::F32>(hb + Lo::hdOst, kBV * 4, static_cast<const float*>(p.dO) + r0 * kVD + v0,
                          (size_t)p.H * kVD * 4, C, L, kBV * 4);
    }
    if constexpr (CF::F32) {
      copy_block<CF>(hb + Lo::hS0, hsrc + vh * hblock_bytes<CF>(), hblock_bytes<CF>());
      copy_block<CF>(hb + Lo::hdS, dhsrc + vh * hblock_bytes<CF>(), hblock_bytes<CF>());
    } else {
      // swizzled [KD][64] state tiles into the padded operand rows
      for (int e = threadIdx.x; e < 2 * kKD * 8; e += blockDim.x) {
        const int m = e / (kKD * 8), r = (e >> 3) % kKD, g = e & 7;
        cp_async16(reinterpret_cast<OpT*>(hb + (m == 0 ? Lo::hS0 : Lo::hdS)) + r * CF::LDV + 8 * g,
                   (m == 0 ? hsrc : dhsrc) + vh * hblock_bytes<CF>() + tc::sw_off(r, 8 * g, kKD));
      }
    }
  };

  load_raw(ch, rq_, rk_, rg_, rkap_, p, b, h, t0, L);
  const char* rec = static_cast<const char*>(p.rec) + cc * RecOf<CF>::bytes;
  if constexpr (CF::F32) {
    copy_block<CF>(sTb, rec + Rec<CF>::T, Rec<CF>::Q - Rec<CF>::T);
    copy_block<CF>(sQb, rec + Rec<CF>::Q, Rec<CF>::F - Rec<CF>::Q);
  } else {
    // swizzled T and scale*Q into the padded operand rows
    for (int e = threadIdx.x; e < 2 * C * (C / 8); e += blockDim.x) {
      const int m = e / (C * (C / 8)), r = (e / (C / 8)) % C, g = e % (C / 8);
      cp_async16((m == 0 ? sTb : sQb) + r * CF::LDC + 8 * g,
                 rec + (m == 0 ? RecTc<CF>::T : RecTc<CF>::Qq) + tc::sw_off(r, 8 * g, C));
    }
  }
  if constexpr (!CF::F32) cp_async_commit();
  issue_half(0);
  if constexpr (!CF::F32) {
    cp_async_commit();
    cp_async_wait_group<1>();  // raw inputs, T and Q
  }
  __syncthreads();
  prep_chunk<CF, 512>(ch);
  for (int e = threadIdx.x; e < 2 * kKD; e += blockDim.x) cfl[e] = 0.f;
  __syncthreads();
  issue_half(1);  // the raw inputs are consumed
  if constexpr (!CF::F32) cp_async_commit();

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
  const float qscale = CF::F32 ? p.scale : 1.f;  // the bf16 record holds scale * Q

  for (int vh = 0; vh < kVD / kBV; ++vh) {
    const int v0 = vh * kBV;
    char* hb = half_base(vh);
    OpT* sv = reinterpret_cast<OpT*>(hb + Lo::hv);
    OpT* sdO = reinterpret_cast<OpT*>(hb + Lo::hdO);
    OpT* sS0 = reinterpret_cast<OpT*>(hb + Lo::hS0);
    OpT* sdS = reinterpret_cast<OpT*>(hb + Lo::hdS);
    float* dOst = reinterpret_cast<float*>(hb + Lo::hdOst);
    if constexpr (!CF::F32) {
      if (vh == 0) {
        cp_async_wait_group<1>();
      } else {
        cp_async_wait_all();
      }
    }
    __syncthreads();
    if constexpr (!CF::ISO) convert_dO<CF>(sdO, dOst);
    // S0' = fr S0, dS'' = fL dS (the bf16 precision saves unscaled states),
    // and cgl += sum_v S0' dS''  (8 threads per state row)
    for (int grp = threadIdx.x; grp < kKD * (kBV / 8); grp += blockDim.x) {
      const int row = grp >> 3, c8 = (grp & 7) * 8;
      float s0[8], ds[8];
      ld8(s0, sS0 + row * CF::LDV + c8);
      ld8(ds, sdS + row * CF::LDV + c8);
      if constexpr (!CF::F32) {
        const float fr = ch.fr[row], fl = ch.fL[row];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          s0[i] *= fr;
          ds[i] *= fl;
        }
        st8(sS0 + row * CF::LDV + c8, s0);
        st8(sdS + row * CF::LDV + c8, ds);
      }
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = fmaf(s0[i], ds[i], acc);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      if ((grp & 7) == 0) cgl[row] += acc;
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
        sDD[row * CF::LDV + col] = from_f<OpT>(qscale * u[0][nt][e] + a[0][nt][e]);
      });
    }
    __syncthreads();

    // dv = T^T ddelta
    {
      float a[1][NTV][4];
      zero_acc(a);
      wgemm<1, NTV, false, false>(a, sTb, CF::LDC, sDD, CF::LDV, 16 * Iv, nv, 16 * Iv, C);
      for_acc_pairs<1, NTV>(a, 16 * Iv, nv, [&](int, int, int, int row, int col, float x0, float x1) {
        if (row < L) st_pair(p.dv + tok_row(p, b, h, t0 + row) * kVD + v0 + col, x0, x1);
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

  // the raw inputs again, for the final gate mapping (overlaps the post-loop products)
  load_raw(ch, rq_, rk_, rg_, rkap_, p, b, h, t0, L);
  if constexpr (!CF::F32) cp_async_commit();

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
    }
  }
  if (own_tri) {
    for_acc<1, 2>(16 * TI, 16 * TJ, [&](int, int nt, int e, int row, int col) {
      sdQ[row * CF::LDC + col] = from_f<OpT>(col <= row ? p.scale * aDQ[0][nt][e] : 0.f);
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
      sdA[row * CF::LDC + col] = from_f<OpT>(col < row ? -x[0][nt][e] : 0.f);
    });
  }
  __syncthreads();
  if constexpr (!CF::F32) cp_async_wait_all();
  __syncthreads();
  if (ch.fast) {
    wgemm<1, NTK, true, false>(aKr, sdA, CF::LDC, ch.Kc, CF::LDK, 16 * I, n0, 0, 16 * (I + 1));
    wgemm<1, NTK, true, false>(aQr, sdQ, CF::LDC, ch.Kc, CF::LDK, 16 * I, n0, 0, 16 * (I + 1));
    wgemm<1, NTK, false, false>(aKc, sdA, CF::LDC, ch.Kr, CF::LDK, 16 * I, n0, 16 * I, C);
    wgemm<1, NTK, false, false>(aKc, sdQ, CF::LDC, ch.Qr, CF::LDK, 16 * I, n0, 16 * I, C);
  }

  // dKr, dQr, dKc to shared memory (fp32, over the operand buffers, which every
  // warp must be done with); one elementwise pass then maps them back through
  // the gate factors, half a warp per row and 8 channels per thread, so row
  // sums are half-warp shuffles and every store is a whole 16-byte granule.
  __syncthreads();
  constexpr int LDO = Lo::LDO;
  float* sXk = reinterpret_cast<float*>(base + Lo::xk);
  float* sXq = reinterpret_cast<float*>(base + Lo::xq);
  float* sXc = reinterpret_cast<float*>(base + Lo::xc);
  store_acc(sXk, LDO, aKr, 16 * I, n0);
  store_acc(sXq, LDO, aQr, 16 * I, n0);
  store_acc(sXc, LDO, aKc, 16 * I, n0);
  __syncthreads();

  const int c0 = (threadIdx.x & 15) * 8;
#pragma unroll 1
  for (int row = threadIdx.x >> 4; row < C; row += 512 / 16) {
    const bool active = row < L;
    const int r = active ? row : L - 1;  // inactive rows compute on a valid row and store nothing
    float g8[8], k8[8], q8[8], dkh[8], dqh[8], dkap[8], dG[8];
    ld8(g8, ch.g + r * kKD + c0);
    ld8(k8, ch.k + r * kKD + c0);
    ld8(q8, ch.q + r * kKD + c0);
    ld8(dkh, sXk + r * LDO + c0);
    ld8(dqh, sXq + r * LDO + c0);
    ld8(dkap, sXc + r * LDO + c0);
    float be = 1.f, rk = 1.f, rq = 1.f;
    if constexpr (CF::ISO) {
      be = ch.beta[r];
      rk = ch.rk[r];
      rq = ch.rq[r];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        k8[i] *= rk;  // k_hat, q_hat
        q8[i] *= rq;
      }
    }
    float kap8[8];
    if constexpr (CF::ISO) {
#pragma unroll
      for (int i = 0; i < 8; ++i) kap8[i] = be * k8[i];
    } else {
      ld8(kap8, ch.kap + r * kKD + c0);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int cu = c0 + i;
      const float rr = ch.fast ? ch.gmid[cu] : 0.f;
      const float rc = ch.fast ? ch.gmid[cu] : ch.glast[cu];
      const float er = ex2a(g8[i] - rr), ec = ex2a(rc - g8[i]);
      const float xk = dkh[i], xq = dqh[i], xc = dkap[i];
      dkh[i] = xk * er;
      dqh[i] = xq * er;
      dkap[i] = xc * ec;
      dG[i] = xk * k8[i] * er + xq * q8[i] * er - xc * kap8[i] * ec;
      // the last row's state term: cgl (formed with S0' = fr S0, dS'' = fL dS)
      // times 2^g_L / (fr fL) = 2^(rc - rr), which stays finite when the three
      // factors underflow (a chunk whose total decay passes 2^-149)
      if (r == L - 1) dG[i] += cfl[cu] + cgl[cu] * ex2(rc - rr);
    }
    if (!ch.fast) {
      // exact gate factors for the score terms
#pragma unroll 1
      for (int j = 0; j < L; ++j) {
        float gj[8], kj[8], qj[8], cj[8];
        ld8(gj, ch.g + j * kKD + c0);
        ld8(kj, ch.k + j * kKD + c0);
        ld8(qj, ch.q + j * kKD + c0);
        if constexpr (CF::ISO) {
          const float rkj = ch.rk[j], rqj = ch.rq[j], bj = ch.beta[j];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            kj[i] *= rkj;
            qj[i] *= rqj;
            cj[i] = bj * kj[i];
          }
        } else {
          ld8(cj, ch.kap + j * kKD + c0);
        }
        const float dAij = j < r ? to_f(sdA[r * CF::LDC + j]) : 0.f;
        const float dQij = j <= r ? to_f(sdQ[r * CF::LDC + j]) : 0.f;
        const float dAji = j > r ? to_f(sdA[j * CF::LDC + r]) : 0.f;
        const float dQji = j >= r ? to_f(sdQ[j * CF::LDC + r]) : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (j <= r) {
            const float f = ex2(g8[i] - gj[i]);
            dkh[i] = fmaf(dAij * cj[i], f, dkh[i]);
            dqh[i] = fmaf(dQij * cj[i], f, dqh[i]);
            dG[i] = fmaf((dAij * k8[i] + dQij * q8[i]) * cj[i], f, dG[i]);
          }
          if (j >= r) {
            const float f = ex2(gj[i] - g8[i]);
            const float w = (dAji * kj[i] + dQji * qj[i]) * f;
            dkap[i] += w;
            dG[i] -= w * kap8[i];
          }
        }
      }
    }
    const size_t off = tok_row(p, b, h, t0 + r) * kKD + c0;
    if (active) st8(p.dg + off, dG);
    if constexpr (CF::ISO) {
      // kappa = beta k_hat: dbeta = <dkappa, k_hat>; then the L2-norm VJPs
      float db = 0.f, dk_dot = 0.f, dq_dot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        db = fmaf(dkap[i], k8[i], db);
        dkh[i] = fmaf(be, dkap[i], dkh[i]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dk_dot = fmaf(dkh[i], k8[i], dk_dot);
        dq_dot = fmaf(dqh[i], q8[i], dq_dot);
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        db += __shfl_xor_sync(0xffffffffu, db, o);
        dk_dot += __shfl_xor_sync(0xffffffffu, dk_dot, o);
        dq_dot += __shfl_xor_sync(0xffffffffu, dq_dot, o);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dkh[i] = rk * (dkh[i] - k8[i] * dk_dot);
        dqh[i] = rq * (dqh[i] - q8[i] * dq_dot);
      }
      if (active) {
        st8(p.dk + off, dkh);
        st8(p.dq + off, dqh);
        if (c0 == 0) p.dbeta[tok_row(p, b, h, t0 + r)] = db;
      }
    } else {
      if (active) {
        st8(p.dkappa + off, dkap);
        st8(p.dk + off, dkh);
        st8(p.dq + off, dqh);
      }
    }
  }
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

template <class CF> int launch_bwd_chunk_tc(const ScanParams&, cudaStream_t);

// The reverse state sweep over chunks [p.c_lo, p.c_hi) (the whole sequence
// for the fp32 precision).
template <class CF>
int launch_bwd_state(const ScanParams& p, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    if constexpr (!CF::F32) {
      if (cudaFuncSetAttribute(scan_bwd_state_tc_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)StateTcLayout<CF>::bytes) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(scan_bwd_state_tc_kernel)");
    }
    configured = true;
  }
  if constexpr (CF::F32) {
    scan_bwd_state_kernel<CF><<<dim3(kVD / kBV, p.B * p.H), kSeqThreads, 0, st>>>(p);
  } else {
    TcMaps maps;
    int rc = CF::ISO ? encode_bthd(&maps.in, p.dO, true, p.B, p.T, p.H, kVD, 64, CF::C, true)
                     : encode_bthd(&maps.in, p.dO, false, p.B, p.T, p.H, kVD, 64, CF::C, false);
    if (rc != KDN_OK) return rc;
    maps.out = maps.in;
    scan_bwd_state_tc_kernel<CF><<<dim3(seq_streams(p), 2), kTcThreads, StateTcLayout<CF>::bytes, st>>>(p, maps);
  }
  return check_launch("scan_bwd_state_kernel");
}

// The chunk-parallel gradients of chunks [p.c_lo, p.c_hi).
template <class CF>
int launch_bwd_chunk(const ScanParams& p, cudaStream_t st) {
  if constexpr (!CF::F32) {
    return launch_bwd_chunk_tc<CF>(p, st);
  } else {
    const size_t s2 = CF::F32 ? 0 : ChunkLayout<CF>::bytes;
    static bool configured = false;
    if (!configured) {
      if (cudaFuncSetAttribute(scan_bwd_chunk_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s2) !=
          cudaSuccess)
        return check_launch("cudaFuncSetAttribute(scan_bwd_chunk_kernel)");
      configured = true;
    }
    scan_bwd_chunk_kernel<CF><<<dim3(p.c_hi - p.c_lo, p.B * p.H), 512, s2, st>>>(p);
    return check_launch("scan_bwd_chunk_kernel");
  }
}

template <class CF>
int launch_bwd(const ScanParams& p, cudaStream_t st) {
  int rc = launch_bwd_state<CF>(p, st);
  if (rc != KDN_OK) return rc;
  return launch_bwd_chunk<CF>(p, st);
}

template int launch_bwd_state<Cfg<true, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_bwd_state<Cfg<false, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_bwd<Cfg<true, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_bwd<Cfg<true, 64, float>>(const ScanParams&, cudaStream_t);
template int launch_bwd<Cfg<false, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_bwd<Cfg<false, 32, float>>(const ScanParams&, cudaStream_t);
template size_t state_bytes<Cfg<true, 64, float>>();
template size_t state_bytes<Cfg<false, 32, float>>();
template size_t chunk_bytes<Cfg<true, 64, float>>();
template size_t chunk_bytes<Cfg<false, 32, float>>();
template size_t state_bytes<Cfg<true, 64, bf16>>();
template size_t state_bytes<Cfg<false, 64, bf16>>();
template size_t chunk_bytes<Cfg<true, 64, bf16>>();
template size_t chunk_bytes<Cfg<false, 64, bf16>>();

}  // namespace kdn
