// Chunk-parallel gradients of the memory scan on tcgen05 tensor cores (bf16
// precision, 64-token chunks, both variants).  One CTA (16 warps) per
// (chunk, b*h).  All operands are
// 128-byte-swizzled bf16 tiles in shared memory (kdn_tc.cuh): the chunk
// record blocks and the saved states arrive by bulk copies, v and dO by TMA,
// the gated operands Kr, Qr, Kc are built from the raw rows in HBM.  Thread 0
// issues six groups of MMAs into tensor memory (512 columns):
//   A  delta^T  = v^T T^T - S0^T Wf^T,  ddelta^T = dO^T Qq + dS''^T Kc^T
//   B  dv = T^T ddelta,  (S0' dO^T, S0' ddelta^T, dS'' delta^T)  [K x C],
//      dO delta^T, ddelta v^T  [C x C]
//   C  dKr^T = dW^T ... (T^T dW)^T,  dT += dW Kr^T
//   D  X = dT T^T      E  dA = -T^T X
//   F  the score terms dA Kc, dQ Kc, dA^T Kr, dQ^T Qr (fast path)
// and the warps turn accumulators into the next operand tiles in between
// (S0' = fr S0, dS'' = fL dS, masks, signs).  The key-side accumulators are
// kept transposed (lane = key), so the final gate mapping has one key per
// lane and every store of a token row is contiguous.  Same mathematics as
// scan_bwd_chunk_kernel (kdn_scan_bwd.cu); replaces _chunk_kda_bwd_precum
// (lit_gpt/kdn_ops/iso_kdn_chunk.py:2089-2187) and the backward of
// _DiagKdnMemoryFunction (diag_kdn_chunk.py:3258-3312).  The diagonal
// variant differs in the gate mapping only (kappa is an input, q and k are
// used as given, dkappa is an output, no token sums) and takes its fp32
// cotangent through the threads, rounded to bf16 as the reference does
// (diag_kdn_chunk.py:3277).
#include "kdn_scan.cuh"
#include "kdn_tc.cuh"
#include "kdn_tma.cuh"

namespace kdn {

struct alignas(64) ChunkMaps {
  CUtensorMap v, dO, dv;  // value rows (128-byte swizzle), dv rows (plain)
  CUtensorMap g, k, q;    // the chunk's raw rows again, plain, for the gate mapping
  CUtensorMap dk, dq, dg; // gradient rows (plain), stored from their staging tiles
};

template <class CF>
struct ChunkTcLayout {
  static_assert(CF::C == 64 && !CF::F32, "bf16 chunks of 64");
  static constexpr int C = 64;
  // whole kernel
  static constexpr size_t Kr = 0, Qr = 16384, Kc = 32768, T = 49152, Xs = 57344;  // Xs: 8 KB scratch
  // the record tiles Qt, Wf and the delta tiles
  static constexpr size_t G = 65536;
  // Qt | delta^T | Wf, then ddelta^T over Wf once the delta products are done
  // (delta^T, ddelta^T: [128 values][C tokens], 128 rows of one 64-column block)
  static constexpr size_t Qt = G, Wf = G + 8192 + 16384;
  static constexpr size_t Del = G + 8192, DDel = Wf;
  // v | dO, then the dv rows, then the raw k | q rows of the gate mapping
  static constexpr size_t V = G + 40960;
  static constexpr size_t vv = V, dO = V + 16384, dvst = V, rk = V, rq = V + 16384;
  static constexpr size_t rg = G;  // raw g rows [C][KD] fp32 over delta | ddelta
  // isotropic: the raw q, k, g rows of the operand build, staged by TMA with
  // the other inputs (g under Kr | Qr, k under Kc, q under delta; read before
  // any of those tiles is written)
  static constexpr size_t sg = Kr, sk = Kc, sq = Del;
  // S0 | dS (saved states), then dW^T dQ dQu dT X dA
  static constexpr size_t A = V + 32768;
  static constexpr size_t S0 = A, dS = A + 32768;
  static constexpr size_t dW = A, dQ = A + 16384, dQu = A + 24576, dT = A + 32768, X = A + 40960, dA = A + 49152;
  // chunk scalars; cfl, cgl [KD]; token sums dbeta, <dk_hat,k_hat>, <dq_hat,q_hat> [C]
  static constexpr size_t small = A + 65536;
  static constexpr size_t bar = small + align_up((small_floats<CF>() + 2 * kKD + 3 * C) * 4, 128);
  static constexpr size_t bytes = bar + 64 + 1024;
  // T, Qt | Wf | S0, dS | v (and dO: the isotropic cotangent arrives by TMA)
  static constexpr unsigned load_bytes = 2 * C * 128 + C * 256 + 2 * 32768 + (CF::ISO ? 2 : 1) * C * 256;
};

// Exact-path score terms of one (token r, key) element: the sum over the
// chunk's other tokens j of dA, dQ times the gate factor 2^(g_r - g_j) (j <= r)
// or 2^(g_j - g_r) (j >= r), each <= 1 (see scan_bwd_chunk_kernel).
struct ExactTerms {
  float dkh, dqh, dkap, dG;
};
// gk: beta rows (isotropic, kappa = beta k_hat) or kappa rows (diagonal)
template <bool ISO>
__device__ __noinline__ ExactTerms exact_terms(const float* g, const bf16* k, const bf16* qv, const float* gk,
                                              const float* rk, const float* rq, int ldr, int ldb, const char* sdA,
                                              const char* sdQ, int r, int key, int L, float gi, float k1, float q1,
                                              float kap) {
  ExactTerms t{0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < L; ++j) {
    const size_t oj = (size_t)j * ldr + key;
    const float gj = g[oj];
    const float khj = (ISO ? rk[j] : 1.f) * __bfloat162float(k[oj]), qhj = (ISO ? rq[j] : 1.f) * __bfloat162float(qv[oj]);
    const float kapj = ISO ? gk[(size_t)j * ldb] * khj : gk[oj];
    if (j <= r) {
      const float f = exp2f(gi - gj);
      const float dAij = j < r ? __bfloat162float(*reinterpret_cast<const bf16*>(sdA + tc::sw_off(r, j, 64))) : 0.f;
      const float dQij = __bfloat162float(*reinterpret_cast<const bf16*>(sdQ + tc::sw_off(r, j, 64)));
      t.dkh = fmaf(dAij * kapj, f, t.dkh);
      t.dqh = fmaf(dQij * kapj, f, t.dqh);
      t.dG = fmaf((dAij * k1 + dQij * q1) * kapj, f, t.dG);
    }
    if (j >= r) {
      const float f = exp2f(gj - gi);
      const float dAji = j > r ? __bfloat162float(*reinterpret_cast<const bf16*>(sdA + tc::sw_off(j, r, 64))) : 0.f;
      const float dQji = __bfloat162float(*reinterpret_cast<const bf16*>(sdQ + tc::sw_off(j, r, 64)));
      const float w = (dAji * khj + dQji * qhj) * f;
      t.dkap += w;
      t.dG -= w * kap;
    }
  }
  return t;
}

// Rows [0, L) of a plain staging tile (row pitch `src_row` bytes) to
// global rows `dst_pitch` bytes apart, 16 bytes per thread and step (every
// thread of the block takes part).
__device__ __forceinline__ void copy_rows_out(void* dst, size_t dst_pitch, const void* src, int src_row, int L) {
  const int g = src_row / 16;
  for (int e = threadIdx.x; e < L * g; e += blockDim.x) {
    const int r = e / g, x = e - r * g;
    *reinterpret_cast<uint4*>(static_cast<char*>(dst) + r * dst_pitch + 16 * x) =
        *reinterpret_cast<const uint4*>(static_cast<const char*>(src) + (size_t)r * src_row + 16 * x);
  }
}

template <class CF>
__global__ void __launch_bounds__(512, 1) scan_bwd_chunk_tc_kernel(ScanParams p, const __grid_constant__ ChunkMaps maps) {
  using Lo = ChunkTcLayout<CF>;
  using RT = RecTc<CF>;
  using OpT = typename CF::OpT;
  constexpr int C = Lo::C;
  // TMEM columns
  constexpr uint32_t TDEL = 0, TDD = 64, TQR = 128, TW = 192, TKC = 256, TDQ = 320, TDT = 384, TKR = 448;
  constexpr uint32_t TDV = 0, TX = 0, TDA = 64;
  extern __shared__ __align__(1024) char smem_raw[];
  char* base = align1024(smem_raw);

  const int c = p.c_lo + blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, cg = warp >> 2;  // TMEM lane quadrant, column group
  int t0, L;
  chunk_span<C>(p, c, t0, L);
  // a packed sequence's last chunk: its boxes ran into the next sequence's
  // rows (zeroed after landing) and its rows leave by plain stores
  const bool tail = p.vl.on() && L < C;
  const size_t cc = (size_t)bh * p.NT + c;
  uint64_t* ldbar = reinterpret_cast<uint64_t*>(base + Lo::bar);
  uint64_t* mmab = ldbar + 1;
  uint64_t* rawbar = ldbar + 2;  // the raw rows of the gate mapping
  // the ddelta products: their own barrier, since both phase-A commits can land
  // before the first wait (one barrier would then have moved two phases on)
  uint64_t* ddbar = ldbar + 3;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(ldbar + 4);
  uint64_t* stbar = ldbar + 5;  // the staged raw rows (isotropic)
  float* small = reinterpret_cast<float*>(base + Lo::small);
  float* cfl = small + small_floats<CF>();
  float* cgl = cfl + kKD;
  float* tsum = cgl + kKD;  // [3][C]

  Chunk<CF> ch;
  bind_raw_global(ch, p, b, h, t0);
  ch.L = L;
  bind_small(ch, small);
  ch.Kr = reinterpret_cast<OpT*>(base + Lo::Kr);
  ch.Qr = reinterpret_cast<OpT*>(base + Lo::Qr);
  ch.Kc = reinterpret_cast<OpT*>(base + Lo::Kc);
  auto bf = [&](size_t off) { return reinterpret_cast<bf16*>(base + off); };
  auto at = [&](size_t tile, int row, int col, int rows) { return reinterpret_cast<bf16*>(base + tile + tc::sw_off(row, col, rows)); };

  if (threadIdx.x == 0) {
    mbar_init(ldbar, 1);
    mbar_init(mmab, 1);
    mbar_init(rawbar, 1);
    mbar_init(ddbar, 1);
    mbar_init(stbar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tc::alloc(tslot, 512);
  for (int e = threadIdx.x; e < 2 * kKD + 3 * C; e += 512) cfl[e] = 0.f;
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);  // this warp's lane quadrant

  // the record tiles, the saved states and the value rows (thread 0)
  auto issue_loads = [&]() {
    const char* rec = static_cast<const char*>(p.rec) + cc * RT::bytes;
    const char* hs = static_cast<const char*>(p.h) + cc * 2 * hblock_bytes<CF>();
    const char* dhs = static_cast<const char*>(p.dh) + cc * 2 * hblock_bytes<CF>();
    mbar_expect_tx(ldbar, Lo::load_bytes);
    bulk_g2s(base + Lo::T, rec + RT::T, C * 128, ldbar);
    bulk_g2s(base + Lo::Qt, rec + RT::Qt, C * 128, ldbar);
    bulk_g2s(base + Lo::Wf, rec + RT::Wf, C * 256, ldbar);
    bulk_g2s(base + Lo::S0, hs, 32768, ldbar);
    bulk_g2s(base + Lo::dS, dhs, 32768, ldbar);
    tma_load_4d(base + Lo::vv, &maps.v, 0, h, t0, b, ldbar);
    tma_load_4d(base + Lo::vv + C * 128, &maps.v, 64, h, t0, b, ldbar);
    if constexpr (CF::ISO) {
      tma_load_4d(base + Lo::dO, &maps.dO, 0, h, t0, b, ldbar);
      tma_load_4d(base + Lo::dO + C * 128, &maps.dO, 64, h, t0, b, ldbar);
    }
  };
  if constexpr (CF::ISO) {
    // every input in flight at once: the raw rows on their own barrier, so the
    // operand build starts as soon as they have landed
    if (threadIdx.x == 0) {
      mbar_expect_tx(stbar, C * kKD * 8);
      tma_load_4d(base + Lo::sg, &maps.g, 0, h, t0, b, stbar);
      tma_load_4d(base + Lo::sk, &maps.k, 0, h, t0, b, stbar);
      tma_load_4d(base + Lo::sq, &maps.q, 0, h, t0, b, stbar);
      issue_loads();
    }
    Chunk<CF> src = ch;
    src.g = reinterpret_cast<const float*>(base + Lo::sg);
    src.k = reinterpret_cast<const bf16*>(base + Lo::sk);
    src.q = reinterpret_cast<const bf16*>(base + Lo::sq);
    src.ldr = kKD;
    prep_chunk<CF, 512, true, true>(ch, &src, stbar, p.status);
  } else {
    // diagonal: the operand build from the rows in HBM first, then the bulk
    // copies (its kappa rows and fp32 cotangent also come through the threads,
    // and staging q, k, g measured slower here: 0.807 against 0.842 ms for
    // kdn_scan_bwd at config 2)
    prep_chunk<CF, 512, true>(ch);
    if (threadIdx.x == 0) issue_loads();
  }
  if constexpr (!CF::ISO) {
    // the fp32 cotangent rounded to bf16 into the swizzled operand tile (rows
    // past the chunk's end zero)
    const float* dO = static_cast<const float*>(p.dO) + tok_row(p, b, h, t0) * kVD;
    for (int e = threadIdx.x; e < C * 16; e += 512) {
      const int r = e >> 4, c8 = 8 * (e & 15);
      float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (r < L) ld8(x, dO + (size_t)r * p.H * kVD + c8);
      *reinterpret_cast<uint4*>(base + Lo::dO + tc::sw_off(r, c8, C)) = pack8(x);
    }
  }
  mbar_wait(ldbar, 0, p.status);
  if (tail) {
    zero_tail_rows<C>(base + Lo::vv, L, threadIdx.x, 512);
    zero_tail_rows<C>(base + Lo::vv + C * 128, L, threadIdx.x, 512);
    if constexpr (CF::ISO) {
      zero_tail_rows<C>(base + Lo::dO, L, threadIdx.x, 512);
      zero_tail_rows<C>(base + Lo::dO + C * 128, L, threadIdx.x, 512);
    }
  }
  fence_async_shared();
  tc::fence_before();
  __syncthreads();

  uint32_t mph = 0;
  auto mma_wait = [&]() {
    mbar_wait(mmab, mph, p.status);
    mph ^= 1;
    tc::fence_after();
  };
  auto publish = [&]() {
    fence_async_shared();
    tc::fence_before();
    __syncthreads();
  };

  float xrow[16];
  // ---- A: delta^T, then ddelta^T (lane = value channel).  The delta products
  // run while the threads scale dS in place (dS'' = fL dS, so Kc replaces
  // the record's Kf = fL Kc); the ddelta products run while they read delta
  // out and scale S0 in place (S0' = fr S0, no longer read by then).
  if (threadIdx.x == 0) {
    tc::fence_after();
    constexpr uint32_t id = tc::idesc(128, C, true, false), idn = tc::idesc(128, C, true, false, true);
    for (int ks = 0; ks < C / 16; ++ks)
      tc::mma(tmem + TDEL, tc::desc_mn(base + Lo::vv, C, ks), tc::desc_k(base + Lo::T, C, ks), id, ks > 0);
    for (int ks = 0; ks < kKD / 16; ++ks)
      tc::mma(tmem + TDEL, tc::desc_mn(base + Lo::S0, kKD, ks), tc::desc_k(base + Lo::Wf, C, ks), idn, true);
    tc::commit(mmab);
  }
  for (int e = threadIdx.x; e < kKD * 16; e += 512) {
    const int r = e >> 4, g = e & 15;
    bf16* ds = at(Lo::dS, r, 8 * g, kKD);
    float d[8];
    ld8(d, ds);
    const float fl = ch.fL[r];
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] *= fl;
    st8(ds, d);
  }
  publish();
  if (threadIdx.x == 0) {
    tc::fence_after();
    constexpr uint32_t id = tc::idesc(128, C, true, false);
    for (int ks = 0; ks < C / 16; ++ks)
      tc::mma(tmem + TDD, tc::desc_mn(base + Lo::dO, C, ks), tc::desc_k(base + Lo::Qt, C, ks), id, ks > 0);
    for (int ks = 0; ks < kKD / 16; ++ks)
      tc::mma(tmem + TDD, tc::desc_mn(base + Lo::dS, kKD, ks), tc::desc_k(base + Lo::Kc, C, ks), id, true);
    tc::commit(ddbar);
  }
  mma_wait();  // delta^T done: S0 and Wf are free
  // delta^T -> bf16 tile [128 values][C tokens]: row v, 16 tokens per thread
  tc::ld16(tq + TDEL + 16 * cg, xrow);
  tc::st_row16(base + Lo::Del, kVD, 32 * q + lane, 16 * cg, xrow, 1.f);
  // S0' = fr S0 in place, cgl = sum_v S0' dS''  (a half-warp per key row)
  for (int e = threadIdx.x; e < kKD * 16; e += 512) {
    const int r = e >> 4, g = e & 15;
    bf16* s0 = at(Lo::S0, r, 8 * g, kKD);
    float a[8], d[8];
    ld8(a, s0);
    ld8(d, at(Lo::dS, r, 8 * g, kKD));
    const float fr = ch.fr[r];
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a[i] *= fr;
      acc = fmaf(a[i], d[i], acc);
    }
    st8(s0, a);
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (g == 0) cgl[r] = acc;
  }
  mbar_wait(ddbar, 0, p.status);  // ddelta^T done
  tc::fence_after();
  tc::ld16(tq + TDD + 16 * cg, xrow);
  tc::st_row16(base + Lo::DDel, kVD, 32 * q + lane, 16 * cg, xrow, 1.f);
  publish();

  // ---- B
  if (threadIdx.x == 0) {
    tc::fence_after();
    // Del, DDel hold delta^T, ddelta^T [values][tokens]
    constexpr uint32_t id_dv = tc::idesc(64, 128, true, false);
    for (int ks = 0; ks < C / 16; ++ks)
      tc::mma(tmem + TDV, tc::desc_mn(base + Lo::T, C, ks), tc::desc_k(base + Lo::DDel, kVD, ks), id_dv, ks > 0);
    constexpr uint32_t id_kc = tc::idesc(128, C, false, false), id_kt = tc::idesc(128, C, false, true);
    constexpr uint32_t id_ct = tc::idesc(64, C, false, true), id_tc = tc::idesc(64, C, true, false);
    for (int ks = 0; ks < kVD / 16; ++ks) {
      tc::mma(tmem + TQR, tc::desc_k(base + Lo::S0, kKD, ks), tc::desc_k(base + Lo::dO, C, ks), id_kc, ks > 0);
      tc::mma(tmem + TW, tc::desc_k(base + Lo::S0, kKD, ks), tc::desc_mn(base + Lo::DDel, kVD, ks), id_kt, ks > 0);
      tc::mma(tmem + TKC, tc::desc_k(base + Lo::dS, kKD, ks), tc::desc_mn(base + Lo::Del, kVD, ks), id_kt, ks > 0);
      tc::mma(tmem + TDQ, tc::desc_k(base + Lo::dO, C, ks), tc::desc_mn(base + Lo::Del, kVD, ks), id_ct, ks > 0);
      tc::mma(tmem + TDT, tc::desc_mn(base + Lo::DDel, kVD, ks), tc::desc_k(base + Lo::vv, C, ks), id_tc, ks > 0);
    }
    tc::commit(mmab);
  }
  mma_wait();
  {
    // dv rows (M = 64 accumulator: row m in lane (m % 16) + 32 (m / 16))
    bf16* dvst = bf(Lo::dvst);
    const int m = 16 * q + (lane & 15);
#pragma unroll
    for (int j = 0; j < 32; j += 16) {
      float x[16];
      tc::ld16(tq + TDV + 32 * cg + j, x);
      if (lane < 16) {
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = x[i];
        st8(dvst + m * kVD + 32 * cg + j, y);
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = x[8 + i];
        st8(dvst + m * kVD + 32 * cg + j + 8, y);
      }
    }
    // dW = -(S0' ddelta^T)^T (lane = key), stored as dW^T [128 keys][C tokens]:
    // row key, 16 tokens per thread
    const int key = 32 * q + lane;
    float x[16];
    tc::ld16(tq + TW + 16 * cg, x);
    tc::st_row16(base + Lo::dW, kKD, key, 16 * cg, x, -1.f);
    // cfl[key] = sum_j Kc[j][key] (delta dS''^T)[j][key]
    tc::ld16(tq + TKC + 16 * cg, x);
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) part = fmaf(to_f(*at(Lo::Kc, 16 * cg + i, key, C)), x[i], part);
    atomicAdd(&cfl[key], part);
    // dQ = scale * lower(dO delta^T) and its unscaled copy
    tc::ld16(tq + TDQ + 16 * cg, x);
    if (lane < 16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = 16 * cg + i <= m ? x[i] : 0.f;
      tc::st_row16(base + Lo::dQu, C, m, 16 * cg, x, 1.f);
      tc::st_row16(base + Lo::dQ, C, m, 16 * cg, x, p.scale);
    }
  }
  publish();
  if (tail) {
    copy_rows_out(p.dv + tok_row(p, b, h, t0) * kVD, (size_t)p.H * kVD * 2, base + Lo::dvst, kVD * 2, L);
  } else if (threadIdx.x == 0) {
    tc::tma_store_4d(&maps.dv, base + Lo::dvst, 0, h, t0, b);
    bulk_commit();
  }

  // ---- C: dKr^T = dW^T T (T read MN-major as the transposed operand), dT += dW Kr^T
  if (threadIdx.x == 0) {
    tc::fence_after();
    constexpr uint32_t id_kr = tc::idesc(128, C, false, true);
    for (int ks = 0; ks < C / 16; ++ks)
      tc::mma(tmem + TKR, tc::desc_k(base + Lo::dW, kKD, ks), tc::desc_mn(base + Lo::T, C, ks), id_kr, ks > 0);
    constexpr uint32_t id_cc = tc::idesc(64, C, true, false);
    for (int ks = 0; ks < kKD / 16; ++ks)
      tc::mma(tmem + TDT, tc::desc_mn(base + Lo::dW, kKD, ks), tc::desc_k(base + Lo::Kr, C, ks), id_cc, true);
    tc::commit(mmab);
    // the delta tiles are dead: the raw g rows of the gate mapping come back meanwhile
    mbar_expect_tx(rawbar, C * kKD * 8);
    tma_load_4d(base + Lo::rg, &maps.g, 0, h, t0, b, rawbar);
  }
  mma_wait();
  auto cc_tile = [&](uint32_t col, size_t tile, float sign, bool strict) {
    // M = 64 accumulator -> masked (j < i, or j <= i) bf16 tile
    float x[16];
    tc::ld16(tq + col + 16 * cg, x);
    if (lane < 16) {
      // this thread's 16 columns of row m are two whole 16-byte granules
      const int m = 16 * q + lane;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = 16 * cg + i;
        x[i] = (strict ? j < m : j <= m) ? x[i] : 0.f;
      }
      tc::st_row16(base + tile, C, m, 16 * cg, x, sign);
    }
  };
  cc_tile(TDT, Lo::dT, 1.f, true);
  publish();
  // ---- D: X = dT T^T
  if (threadIdx.x == 0) {
    tc::fence_after();
    constexpr uint32_t id_cc = tc::idesc(64, C, false, false);
    for (int ks = 0; ks < C / 16; ++ks)
      tc::mma(tmem + TX, tc::desc_k(base + Lo::dT, C, ks), tc::desc_k(base + Lo::T, C, ks), id_cc, ks > 0);
    tc::commit(mmab);
    // ... and the raw k, q rows over the value tiles once the dv rows have left
    bulk_wait_read<0>();
    tma_load_4d(base + Lo::rk, &maps.k, 0, h, t0, b, rawbar);
    tma_load_4d(base + Lo::rq, &maps.q, 0, h, t0, b, rawbar);
  }
  mma_wait();
  cc_tile(TX, Lo::X, 1.f, true);
  publish();
  // ---- E: dA = -T^T X (strictly lower)
  if (threadIdx.x == 0) {
    tc::fence_after();
    constexpr uint32_t id_cc = tc::idesc(64, C, true, true);
    for (int ks = 0; ks < C / 16; ++ks)
      tc::mma(tmem + TDA, tc::desc_mn(base + Lo::T, C, ks), tc::desc_mn(base + Lo::X, C, ks), id_cc, ks > 0);
    tc::commit(mmab);
  }
  mma_wait();
  cc_tile(TDA, Lo::dA, -1.f, true);
  publish();
  // ---- F: score terms (the exact path adds them elementwise below)
  if (ch.fast) {
    if (threadIdx.x == 0) {
      tc::fence_after();
      constexpr uint32_t id_t = tc::idesc(128, C, true, false), id_n = tc::idesc(128, C, true, true);
      for (int ks = 0; ks < C / 16; ++ks) {
        tc::mma(tmem + TKR, tc::desc_mn(base + Lo::Kc, C, ks), tc::desc_k(base + Lo::dA, C, ks), id_t, true);
        tc::mma(tmem + TQR, tc::desc_mn(base + Lo::Kc, C, ks), tc::desc_k(base + Lo::dQu, C, ks), id_t, true);
        tc::mma(tmem + TKC, tc::desc_mn(base + Lo::Kr, C, ks), tc::desc_mn(base + Lo::dA, C, ks), id_n, true);
      }
      for (int ks = 0; ks < C / 16; ++ks)
        tc::mma(tmem + TKC, tc::desc_mn(base + Lo::Qr, C, ks), tc::desc_mn(base + Lo::dQ, C, ks), id_n, true);
      tc::commit(mmab);
    }
    mma_wait();
  }

  // ---- gate mapping: lane = key, 16 tokens per thread
  mbar_wait(rawbar, 0, p.status);
  const int key = 32 * q + lane;
  float xk[16], xq[16], xc[16];
  tc::ld16(tq + TKR + 16 * cg, xk);
  tc::ld16(tq + TQR + 16 * cg, xq);
  tc::ld16(tq + TKC + 16 * cg, xc);
  const float rr = ch.fast ? ch.gmid[key] : 0.f;
  const float rc = ch.fast ? ch.gmid[key] : ch.glast[key];
  // the last row's state term: cgl was formed with S0' = fr S0 and dS'' = fL dS,
  // so it carries 2^g_L / (fr fL) = 2^(rc - rr) (1 on the fast path); taken as
  // that power so it stays finite when 2^g_L, fr and fL all underflow (a chunk
  // whose total decay passes 2^-149 while its range around rho stays small)
  const float last = cfl[key] + cgl[key] * ex2(rc - rr);
  float* part = reinterpret_cast<float*>(base + Lo::X);  // [4 quadrants][3][C] partial token sums
  // exact-path terms of 8 tokens per thread, [8][4][512] fp32 over the operand
  // tiles Kr .. Xs (dead once the score MMAs are skipped)
  float* xs = reinterpret_cast<float*>(base + Lo::Kr);
  static_assert(Lo::Xs + 8192 >= 8 * 4 * 512 * 4, "exact-path scratch");
  // the same 64 KB once the mapping is done (on the fast path already during
  // it): the dg, dk, dq rows [C][128], written lane = key and stored by TMA
  float* sdg = xs;
  bf16* sdk = reinterpret_cast<bf16*>(base + Lo::Kr + C * kKD * 4);
  bf16* sdq = sdk + C * kKD;
  static_assert(Lo::Kr + C * kKD * 8 <= Lo::Xs + 8192, "output staging");
  float kh[16], qh[16];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    if (!ch.fast) {
#pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        const int tok = 16 * cg + 8 * half + i;
        const int r = tok < L ? tok : L - 1;
        const size_t off = (size_t)r * ch.ldr + key;
        const float gi = ch.g[off];
        ExactTerms t;
        if constexpr (CF::ISO) {
          const float k1 = ch.rk[r] * to_f(ch.k[off]), q1 = ch.rq[r] * to_f(ch.q[off]);
          const float kap = ch.beta[(size_t)r * ch.ldb] * k1;
          t = exact_terms<true>(ch.g, ch.k, ch.q, ch.beta, ch.rk, ch.rq, ch.ldr, ch.ldb, base + Lo::dA, base + Lo::dQ,
                                r, key, L, gi, k1, q1, kap);
        } else {
          t = exact_terms<false>(ch.g, ch.k, ch.q, ch.kap, nullptr, nullptr, ch.ldr, ch.ldb, base + Lo::dA,
                                 base + Lo::dQ, r, key, L, gi, to_f(ch.k[off]), to_f(ch.q[off]), ch.kap[off]);
        }
        xs[(i * 4 + 0) * 512 + threadIdx.x] = t.dkh;
        xs[(i * 4 + 1) * 512 + threadIdx.x] = t.dqh;
        xs[(i * 4 + 2) * 512 + threadIdx.x] = t.dkap;
        xs[(i * 4 + 3) * 512 + threadIdx.x] = t.dG;
      }
    }
    // raw rows of 8 tokens (shared memory; kappa from global), then the arithmetic
    float gv[8], kv[8], qv[8], kapv[CF::ISO ? 1 : 8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int tok = 16 * cg + 8 * half + i;
      const int r = tok < L ? tok : L - 1;
      if constexpr (!CF::ISO) kapv[i] = ch.kap[(size_t)r * ch.ldr + key];
      gv[i] = reinterpret_cast<const float*>(base + Lo::rg)[r * kKD + key];
      kv[i] = to_f(bf(Lo::rk)[r * kKD + key]);
      qv[i] = to_f(bf(Lo::rq)[r * kKD + key]);
    }
    float dgv[8], db[8], dkd[8], dqd[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int ii = 8 * half + i;
      const int tok = 16 * cg + ii;
      const int r = tok < L ? tok : L - 1;
      float k1, q1, kap, be = 0.f;
      if constexpr (CF::ISO) {
        be = ch.rb[r];
        k1 = ch.rk[r] * kv[i];
        q1 = ch.rq[r] * qv[i];
        kap = be * k1;
      } else {
        k1 = kv[i];
        q1 = qv[i];
        kap = kapv[i];
      }
      const float gi = gv[i];
      const float er = ex2a(gi - rr), ec = ex2a(rc - gi);
      const float dKr = xk[ii], dQr = p.scale * xq[ii], dKc = xc[ii];
      float dkh = dKr * er, dqh = dQr * er, dkap = dKc * ec;
      float dG = dKr * k1 * er + dQr * q1 * er - dKc * kap * ec;
      if (r == L - 1) dG += last;
      if (!ch.fast) {
        dkh += xs[(i * 4 + 0) * 512 + threadIdx.x];
        dqh += xs[(i * 4 + 1) * 512 + threadIdx.x];
        dkap += xs[(i * 4 + 2) * 512 + threadIdx.x];
        dG += xs[(i * 4 + 3) * 512 + threadIdx.x];
      }
      dgv[i] = dG;
      if constexpr (CF::ISO) {
        db[i] = dkap * k1;          // dbeta = <dkappa, k_hat>
        dkh = fmaf(be, dkap, dkh);  // kappa = beta k_hat
        dkd[i] = dkh * k1;
        dqd[i] = dqh * q1;
      } else {
        db[i] = dkap;  // dkappa itself
        dkd[i] = dqd[i] = 0.f;
      }
      xk[ii] = dkh;
      xq[ii] = dqh;
      kh[ii] = k1;
      qh[ii] = q1;
    }
    if (ch.fast) {
#pragma unroll
      for (int i = 0; i < 8; ++i) sdg[(16 * cg + 8 * half + i) * kKD + key] = dgv[i];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int tok = 16 * cg + 8 * half + i;
        if (tok < L) p.dg[tok_row(p, b, h, t0 + tok) * kKD + key] = dgv[i];
      }
    }
    if constexpr (CF::ISO) {
      // token sums over this warp's 32 keys: one transpose-reduce leaves the sum
      // of value j in lane j (j = 8 * quantity + token)
      float v32[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v32[i] = db[i];
        v32[8 + i] = dkd[i];
        v32[16 + i] = dqd[i];
        v32[24 + i] = 0.f;
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = lane & off;
#pragma unroll
        for (int i = 0; i < off; ++i) {
          const float send = upper ? v32[i] : v32[i + off];
          const float keep = upper ? v32[i + off] : v32[i];
          v32[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      if (lane < 24) part[(q * 3 + (lane >> 3)) * C + 16 * cg + 8 * half + (lane & 7)] = v32[0];
    } else {
      // dkappa rows straight to HBM (128 bytes per warp and token)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int tok = 16 * cg + 8 * half + i;
        if (tok < L) p.dkappa[tok_row(p, b, h, t0 + tok) * kKD + key] = db[i];
      }
    }
  }
  __syncthreads();
  if constexpr (CF::ISO) {
    if (threadIdx.x < 3 * C) {
      const int sidx = threadIdx.x / C, tok = threadIdx.x % C;
      float t = 0.f;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) t += part[(qq * 3 + sidx) * C + tok];
      tsum[threadIdx.x] = t;
    }
    __syncthreads();
    float rkv[16], rqv[16], dkdot[16], dqdot[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int tok = 16 * cg + i;
      rkv[i] = ch.rk[tok];
      rqv[i] = ch.rq[tok];
      dkdot[i] = tsum[C + tok];
      dqdot[i] = tsum[2 * C + tok];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int tok = 16 * cg + i;
      sdk[tok * kKD + key] = __float2bfloat16_rn(rkv[i] * (xk[i] - kh[i] * dkdot[i]));
      sdq[tok * kKD + key] = __float2bfloat16_rn(rqv[i] * (xq[i] - qh[i] * dqdot[i]));
    }
    if (threadIdx.x < L) p.dbeta[tok_row(p, b, h, t0 + threadIdx.x)] = tsum[threadIdx.x];
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int tok = 16 * cg + i;
      sdk[tok * kKD + key] = __float2bfloat16_rn(xk[i]);
      sdq[tok * kKD + key] = __float2bfloat16_rn(xq[i]);
    }
  }
  // the staged rows leave by TMA stores (rows past the sequence's end are clipped)
  fence_async_shared();
  __syncthreads();
  if (tail) {
    const size_t r0 = tok_row(p, b, h, t0);
    copy_rows_out(p.dk + r0 * kKD, (size_t)p.H * kKD * 2, sdk, kKD * 2, L);
    copy_rows_out(p.dq + r0 * kKD, (size_t)p.H * kKD * 2, sdq, kKD * 2, L);
    if (ch.fast) copy_rows_out(p.dg + r0 * kKD, (size_t)p.H * kKD * 4, sdg, kKD * 4, L);
  } else if (threadIdx.x == 0) {
    tc::tma_store_4d(&maps.dk, sdk, 0, h, t0, b);
    tc::tma_store_4d(&maps.dq, sdq, 0, h, t0, b);
    if (ch.fast) tc::tma_store_4d(&maps.dg, sdg, 0, h, t0, b);
    bulk_commit();
  }

  // shared memory must outlive the stores' reads; their writes complete on their own
  if (threadIdx.x == 0) bulk_wait_read<0>();
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::dealloc(tmem, 512);
  }
}

template <class CF>
int launch_bwd_chunk_tc(const ScanParams& p, cudaStream_t st) {
  const size_t smem = ChunkTcLayout<CF>::bytes;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(scan_bwd_chunk_tc_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return check_launch("cudaFuncSetAttribute(scan_bwd_chunk_tc_kernel)");
    configured = true;
  }
  ChunkMaps maps;
  int rc = encode_bthd(&maps.v, p.v, true, p.B, p.T, p.H, kVD, 64, CF::C, true);
  if (rc == KDN_OK && CF::ISO) rc = encode_bthd(&maps.dO, p.dO, true, p.B, p.T, p.H, kVD, 64, CF::C, true);
  if (rc == KDN_OK) rc = encode_bthd(&maps.dv, p.dv, true, p.B, p.T, p.H, kVD, kVD, CF::C, false);
  if (rc == KDN_OK) rc = encode_bthd(&maps.g, p.g, false, p.B, p.T, p.H, kKD, kKD, CF::C, false);
  if (rc == KDN_OK) rc = encode_bthd(&maps.k, p.k, true, p.B, p.T, p.H, kKD, kKD, CF::C, false);
  if (rc == KDN_OK) rc = encode_bthd(&maps.q, p.q, true, p.B, p.T, p.H, kKD, kKD, CF::C, false);
  if (rc == KDN_OK) rc = encode_bthd(&maps.dk, p.dk, true, p.B, p.T, p.H, kKD, kKD, CF::C, false);
  if (rc == KDN_OK) rc = encode_bthd(&maps.dq, p.dq, true, p.B, p.T, p.H, kKD, kKD, CF::C, false);
  if (rc == KDN_OK) rc = encode_bthd(&maps.dg, p.dg, false, p.B, p.T, p.H, kKD, kKD, CF::C, false);
  if (rc != KDN_OK) return rc;
  scan_bwd_chunk_tc_kernel<CF><<<dim3(p.c_hi - p.c_lo, p.B * p.H), 512, smem, st>>>(p, maps);
  return check_launch("scan_bwd_chunk_tc_kernel");
}

template int launch_bwd_chunk_tc<Cfg<true, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_bwd_chunk_tc<Cfg<false, 64, bf16>>(const ScanParams&, cudaStream_t);

}  // namespace kdn
