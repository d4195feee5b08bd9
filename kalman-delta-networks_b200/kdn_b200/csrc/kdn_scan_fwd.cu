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
#include "kdn_tc.cuh"
#include "kdn_tma.cuh"

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

// ---------------------------------------------------------------------------
// Tensor-core sequential pass (bf16 precision): two CTAs per (b, h) stream,
// each carrying 64 value columns of the 128 x 128 fp32 state in TMEM (the
// recurrence does not mix value columns).  Warps 0-7 move data between TMEM
// and shared memory, thread 0 issues the MMAs, warp 8 streams the chunk
// records (bulk copy) and the CTA's value columns (TMA, 128-byte swizzle)
// into NS stages.  Per chunk, with the record's folded factors
// (Qs = scale fr Qr, Kf = fL Kc, Wf = fr W0, Qq = scale Q):
//   S -> bf16 operand (saved as h);  S <- 2^g_L S            (TMEM ld / st)
//   delta^T = v^T T^T - S^T Wf^T                               (MMA, M = 64 values)
//   o^T = S^T Qs^T + delta^T Qq^T;  S += Kf^T delta            (MMA)
//   o -> shared memory -> one TMA store of the chunk's rows
// ---------------------------------------------------------------------------
template <class CF>
struct FwdTcLayout {
  static constexpr int C = CF::C;
  static constexpr int NS = CF::C == 64 ? 2 : 3;
  using R = RecTc<CF>;
  static constexpr size_t v = R::fwd_end;  // [C][64] bf16, swizzled by the TMA engine
  static constexpr size_t stage = align_up(v + (size_t)C * 128, 1024);
  static constexpr size_t S = NS * stage;                 // state operand [KD][64] bf16 (also h)
  static constexpr size_t Del = S + (size_t)kKD * 128;    // delta^T [64][C] bf16
  static constexpr size_t O = Del + (size_t)C * 128;      // output rows [C][64] (bf16 iso, fp32 diag)
  static constexpr size_t O_bytes = (size_t)C * 64 * (CF::ISO ? 2 : 4);
  static constexpr size_t bar = O + align_up(O_bytes, 1024);
  static constexpr size_t bytes = bar + 128 + 1024;       // barriers and TMEM slot; alignment slack
};

template <class CF>
__global__ void __launch_bounds__(kTcThreads, 1) scan_fwd_tc_kernel(ScanParams p, const __grid_constant__ TcMaps maps) {
  using Lo = FwdTcLayout<CF>;
  using R = RecTc<CF>;
  using OutT = typename std::conditional<CF::ISO, bf16, float>::type;
  constexpr int C = CF::C, NS = Lo::NS, HC = C / 2;
  constexpr uint32_t TS = 0, TD = 64, TO = 64 + C;  // TMEM columns: state, delta^T, o^T
  constexpr int NTH = kTcWarps * 32;
  extern __shared__ __align__(1024) char smem_raw[];
  char* base = align1024(smem_raw);

  const SeqStream ss = seq_stream(p, blockIdx.x);
  const int vh = blockIdx.y, V0 = 64 * vh, b = ss.b, h = ss.h, c_lo = ss.c_lo, c_hi = ss.c_hi;
  const bool vl = p.vl.on();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const char* recs = static_cast<const char*>(p.rec) + ss.rec_row * p.NT * R::bytes;
  char* hout = static_cast<char*>(p.h) + ss.rec_row * p.NT * 2 * hblock_bytes<CF>() + (size_t)vh * hblock_bytes<CF>();
  uint64_t* full = reinterpret_cast<uint64_t*>(base + Lo::bar);
  uint64_t* empty = full + NS;
  uint64_t* mmab = empty + NS;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mmab + 1);
  char* sS = base + Lo::S;
  char* sDel = base + Lo::Del;

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

  // state-map mode: blockIdx.z = 1 runs the identity with zero values (no v
  // rows, no delta term from v), and neither run writes o or h
  const bool smap = p.state_map != 0, phi = smap && blockIdx.z == 1;
  if (warp == kTcWarps) {
    // producer: refill a stage once the MMAs of its previous chunk completed
    for (int c = c_lo; c < c_hi; ++c) {
      const int it = c - c_lo, s = it % NS;
      if (it >= NS) mbar_wait(&empty[s], (it / NS - 1) & 1, p.status);
      if (lane == 0) {
        char* st = base + s * Lo::stage;
        int t0, L;
        chunk_span<C>(p, c, t0, L);
        mbar_expect_tx(&full[s], (unsigned)(R::fwd_end + (phi ? 0 : (size_t)C * 128)));
        bulk_g2s(st, recs + (size_t)c * R::bytes, (unsigned)R::fwd_end, &full[s]);
        if (!phi) tma_load_4d(st + Lo::v, &maps.in, V0, h, t0, b, &full[s]);
      }
      __syncwarp();
    }
    return;
  }

  // compute warps: warp w reads TMEM lanes 32(w%4).., column half w/4; the
  // M = 64 accumulators delta^T, o^T hold value column m in lane
  // (m % 16) + 32 (m / 16), i.e. lanes 0-15 of each quadrant
  const int q = warp & 3, hf = warp >> 2;
  const int row = 32 * q + lane;  // key (state)
  const int vc = 16 * q + lane;   // value column of this CTA (delta^T, o^T; lanes < 16)
  const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
  for (int j = 0; j < 32; j += 16) {
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int col = V0 + 32 * hf + j + i;
      x[i] = phi ? (row == col ? 1.f : 0.f) : p.S0 ? p.S0[(ss.state * kKD + row) * kVD + col] : 0.f;
    }
    tc::st16(tl + TS + 32 * hf + j, x);
  }
  tc::wait_st();
  uint32_t mph = 0;

  // Software-pipelined over chunks: chunk c's output rows are read out of
  // TMEM while the delta products of chunk c + 1 run.
  //   head(c):  state operand (and h) from TMEM, S <- 2^g_L S, delta MMAs
  //   body(c):  delta -> operand tile, o and state MMAs, then head(c + 1),
  //             then o(c) -> output tile -> TMA store
  char* sO = base + Lo::O;
  auto head = [&](int c) {
    const int it = c - c_lo, s = it % NS;
    char* st = base + s * Lo::stage;
    mbar_wait(&full[s], (it / NS) & 1, p.status);
    if (vl) {
      // a sequence's last chunk: the box ran into the next sequence's rows
      int t0, L;
      chunk_span<C>(p, c, t0, L);
      if (L < C) zero_tail_rows<C>(st + Lo::v, L, threadIdx.x, NTH);
    }
    const float gl = reinterpret_cast<const float*>(st + R::F)[2 * kKD + row];
#pragma unroll
    for (int j = 0; j < 32; j += 16) {
      float x[16];
      tc::ld16(tl + TS + 32 * hf + j, x);
      tc::st_row16(sS, kKD, row, 32 * hf + j, x, 1.f);
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] *= gl;
      tc::st16(tl + TS + 32 * hf + j, x);
    }
    // (the scaled state's TMEM stores complete before the state MMA: wait_st in the body)
    if (threadIdx.x == 0) bulk_wait_read<0>();  // the previous output rows have left their tile
    fence_async_shared();
    tc::fence_before();
    bar_sync(1, NTH);
    if (threadIdx.x == 32 && !smap) {
      bulk_s2g(hout + (size_t)c * 2 * hblock_bytes<CF>(), sS, (unsigned)hblock_bytes<CF>());
      bulk_commit();
    }
    if (threadIdx.x == 0) {
      tc::fence_after();
      constexpr uint32_t id = tc::idesc(64, C, true, false), idn = tc::idesc(64, C, true, false, true);
      if (!phi)
        for (int ks = 0; ks < C / 16; ++ks)
          tc::mma(tmem + TD, tc::desc_mn(st + Lo::v, C, ks), tc::desc_k(st + R::T, C, ks), id, ks > 0);
      for (int ks = 0; ks < kKD / 16; ++ks)
        tc::mma(tmem + TD, tc::desc_mn(sS, kKD, ks), tc::desc_k(st + R::Wf, C, ks), idn, !phi || ks > 0);
      tc::commit(mmab);
    }
  };

  if (c_lo < c_hi) head(c_lo);
  for (int c = c_lo; c < c_hi; ++c) {
    const int it = c - c_lo, s = it % NS;
    int t0, L;
    chunk_span<C>(p, c, t0, L);
    char* st = base + s * Lo::stage;
    mbar_wait(mmab, mph, p.status);
    mph ^= 1;
    tc::fence_after();
    // delta^T (value row vc, lanes < 16) -> bf16 operand tile [64][C], 16 tokens
    // per two 16-byte stores
#pragma unroll
    for (int j = 0; j < HC; j += 16) {
      float x[16];
      tc::ld16(tl + TD + HC * hf + j, x);
      if (lane < 16) tc::st_row16(sDel, 64, vc, HC * hf + j, x, 1.f);
    }
    if (threadIdx.x == 32) bulk_wait_read<0>();  // h has left the state operand (rewritten next chunk)
    tc::wait_st();
    fence_async_shared();
    tc::fence_before();
    bar_sync(1, NTH);
    if (threadIdx.x == 0) {
      tc::fence_after();
      constexpr uint32_t ido = tc::idesc(64, C, true, false), idd = tc::idesc(64, C, false, false);
      constexpr uint32_t ids = tc::idesc(128, 64, true, false);
      if (!smap) {
        for (int ks = 0; ks < kKD / 16; ++ks)
          tc::mma(tmem + TO, tc::desc_mn(sS, kKD, ks), tc::desc_k(st + R::Qs, C, ks), ido, ks > 0);
        for (int ks = 0; ks < C / 16; ++ks)
          tc::mma(tmem + TO, tc::desc_k(sDel, 64, ks), tc::desc_k(st + R::Qq, C, ks), idd, true);
      }
      for (int ks = 0; ks < C / 16; ++ks)
        tc::mma(tmem + TS, tc::desc_mn(st + R::Kf, C, ks), tc::desc_k(sDel, 64, ks), ids, true);
      tc::commit(&empty[s]);
      tc::commit(mmab);
    }
    mbar_wait(mmab, mph, p.status);
    mph ^= 1;
    tc::fence_after();
    // the next chunk's delta products go first (they write other TMEM columns
    // and no tile this chunk still reads) ...
    if (c + 1 < c_hi) {
      head(c + 1);
    } else {
      if (threadIdx.x == 0) bulk_wait_read<0>();
      bar_sync(1, NTH);
    }
    if (smap) continue;
    // ... then this chunk's output rows (value column vc) into their tile and one TMA store
    {
      OutT* o = reinterpret_cast<OutT*>(sO);
#pragma unroll
      for (int j = 0; j < HC; j += 16) {
        float x[16];
        tc::ld16(tl + TO + HC * hf + j, x);
        if (lane < 16) {
#pragma unroll
          for (int i = 0; i < 16; ++i) o[(HC * hf + j + i) * 64 + vc] = from_f<OutT>(x[i]);
        }
      }
    }
    fence_async_shared();
    tc::fence_before();
    bar_sync(1, NTH);
    if (vl && L < C) {
      // a sequence's last chunk of a packed batch: rows past its end belong
      // to the next sequence, so the rows leave by plain stores
      constexpr int G = 64 * (int)sizeof(OutT) / 16;  // 16-byte granules per row
      for (int e = threadIdx.x; e < L * G; e += NTH) {
        const int r = e / G, gi = e - r * G;
        *reinterpret_cast<uint4*>(static_cast<OutT*>(p.o) + tok_row(p, b, h, t0 + r) * kVD + V0 + gi * (16 / sizeof(OutT))) =
            *reinterpret_cast<const uint4*>(sO + (size_t)r * 64 * sizeof(OutT) + gi * 16);
      }
    } else if (threadIdx.x == 0) {
      tc::tma_store_4d(&maps.out, sO, V0, h, t0, b);
      bulk_commit();
    }
  }
  float* ST = phi ? p.ST2 : p.ST;
  if (ST) {
    for (int j = 0; j < 32; j += 16) {
      float x[16];
      tc::ld16(tl + TS + 32 * hf + j, x);
#pragma unroll
      for (int i = 0; i < 16; ++i) ST[(ss.state * kKD + row) * kVD + V0 + 32 * hf + j + i] = x[i];
    }
  }
  if (threadIdx.x == 0 || threadIdx.x == 32) bulk_wait_all();
  tc::fence_before();
  bar_sync(1, NTH);
  if (warp == 0) {
    tc::fence_after();
    tc::dealloc(tmem, 256);
  }
}

template <class CF>
size_t fwd_dbg_bytes() {
  return CF::F32 ? FwdLayout<CF>::bytes : 0;
}

template <class CF> int launch_prep(const ScanParams&, cudaStream_t);

// The sequential forward pass over chunks [p.c_lo, p.c_hi) (the whole
// sequence for the fp32 precision).
template <class CF>
int launch_fwd_seq(const ScanParams& p, cudaStream_t st) {
  int rc = KDN_OK;
  static bool configured = false;
  if constexpr (CF::F32) {
    if (!configured) {
      if (cudaFuncSetAttribute(scan_fwd_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, 0) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(scan_fwd_kernel)");
      configured = true;
    }
    dim3 grid(kVD / kBV, p.B * p.H);
    scan_fwd_kernel<CF><<<grid, kSeqThreads, 0, st>>>(p);
    return check_launch("scan_fwd_kernel");
  } else {
    const size_t smem = FwdTcLayout<CF>::bytes;
    if (!configured) {
      if (cudaFuncSetAttribute(scan_fwd_tc_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
        return check_launch("cudaFuncSetAttribute(scan_fwd_tc_kernel)");
      configured = true;
    }
    TcMaps maps;
    rc = encode_bthd(&maps.in, p.v, true, p.B, p.T, p.H, kVD, 64, CF::C, true);
    if (rc != KDN_OK) return rc;
    if (p.state_map) {
      maps.out = maps.in;  // no output rows in state-map mode
    } else {
      rc = encode_bthd(&maps.out, p.o, CF::ISO, p.B, p.T, p.H, kVD, 64, CF::C, false);
      if (rc != KDN_OK) return rc;
    }
    scan_fwd_tc_kernel<CF><<<dim3(seq_streams(p), 2, p.state_map ? 2 : 1), kTcThreads, smem, st>>>(p, maps);
    return check_launch("scan_fwd_tc_kernel");
  }
}

template <class CF>
int launch_fwd(const ScanParams& p, cudaStream_t st) {
  int rc = launch_prep<CF>(p, st);
  if (rc != KDN_OK) return rc;
  return launch_fwd_seq<CF>(p, st);
}

template int launch_fwd_seq<Cfg<true, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_fwd_seq<Cfg<false, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<true, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<true, 64, float>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<false, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_fwd<Cfg<false, 32, float>>(const ScanParams&, cudaStream_t);
template size_t fwd_dbg_bytes<Cfg<true, 64, float>>();
template size_t fwd_dbg_bytes<Cfg<false, 32, float>>();

}  // namespace kdn
