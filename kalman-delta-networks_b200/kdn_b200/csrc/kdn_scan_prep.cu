// Chunk-parallel first pass of the chunked KDN memory scan: everything a
// chunk needs that does not depend on the running state.  One CTA per
// (chunk, b*h), two CTAs per SM; the raw rows come straight from HBM.
//   q, k, g, kappa|beta -> gated operands Kr, Qr, Kc (reference rho, exact
//   path for wide gate ranges) -> A = Kr Kc^T, Q = Qr Kc^T (tensor cores)
//   -> T = (I + A)^-1 -> W0 = T Kr
// and writes the chunk record: (Qr, Kc, W0, T, Q, fr, fL, 2^g_L) as padded
// rows in the fp32 precision, or the swizzled tensor-core tiles with the
// scale factors folded in (RecTc) in the bf16 precision.  The sequential forward and reverse passes then
// only carry the state.  Replaces the intra-chunk half of
// _chunk_kda_fwd_precum (lit_gpt/kdn_ops/iso_kdn_chunk.py:2037-2086, the
// scaled-dot-kkt / solve-tril / recompute-w-u stages of the FLA pipeline it
// calls) and of _diag_kdn_memory_forward (diag_kdn_chunk.py:3224-3245).
#include "kdn_scan.cuh"
#include "kdn_tc.cuh"
#include "kdn_tma.cuh"

namespace kdn {

constexpr int kPrepThreads = 256;

// The chunk's raw q, k (bf16) and g (fp32) rows, staged by TMA (bf16
// records): one box of C tokens x 128 channels each.
struct alignas(64) PrepMaps {
  CUtensorMap q, k, g;
};
template <class CF>
__host__ __device__ constexpr bool prep_staged() {
  return !CF::F32;
}

template <class CF>
struct PrepLayout {
  static constexpr size_t sz = sizeof(typename CF::OpT);
  static constexpr int C = CF::C;
  static constexpr size_t Kr = 0;  // holds W0 = T Kr at the end
  static constexpr size_t Qr = Kr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Kc = Qr + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Tb = Kc + A128((size_t)C * CF::LDK * sz);
  static constexpr size_t Qb = Tb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t Xb = Qb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t Ab = Xb + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t As = Ab + A128((size_t)C * CF::LDC * sz);
  static constexpr size_t small = As + A128((size_t)C * CF::LDA * 4);
  static constexpr size_t base_bytes = small + A128(small_floats<CF>() * 4);
  // bf16 record tiles T, Qq, Qt ([C][64] swizzled each), staged for the
  // bulk stores over Xb .. As (dead after the solve) when they fit there
  static constexpr size_t rec_tiles = 3 * (size_t)C * 128;
  static constexpr bool alias = small - Xb >= rec_tiles;
  static constexpr size_t St = alias ? Xb : base_bytes;
  // staged raw rows (prep_staged): k under Kr, q under Qr, g over Tb .. As
  // (their first users come after the operand build)
  static constexpr size_t raw_k = Kr, raw_q = Qr, raw_g = Tb;
  static_assert(raw_g + (size_t)C * kKD * 4 <= small, "raw g rows fit below the chunk scalars");
  static_assert((size_t)C * kKD * 2 <= Qr - Kr, "raw k rows fit under Kr");
  static_assert(raw_q + (size_t)C * kKD * 2 <= Kc && raw_g >= Tb, "no raw row is staged under Kc (prep_chunk stores Kc early)");
  static constexpr size_t bar = (alias ? base_bytes : base_bytes + rec_tiles);
  static constexpr size_t bytes = bar + 16;
};

template <class CF>
__global__ void __launch_bounds__(kPrepThreads, 2) scan_prep_kernel(ScanParams p, const __grid_constant__ PrepMaps maps) {
  using OpT = typename CF::OpT;
  using Lo = PrepLayout<CF>;
  using R = Rec<CF>;
  constexpr int C = CF::C;
  constexpr int NJ = (kPrepThreads / 32) / (C / 16);  // warps per 16-row block of W0
  constexpr int NTW = kKD / (8 * NJ);
  extern __shared__ __align__(128) char smem[];
  char* base = CF::F32 ? p.dbg + (size_t)(blockIdx.y * gridDim.x + blockIdx.x) * p.dbg_stride : smem;

  const int c = p.c_lo + blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int warp = threadIdx.x >> 5;
  int t0, L;
  chunk_span<C>(p, c, t0, L);
  const size_t cc = (size_t)bh * p.NT + c;

  Chunk<CF> ch;
  bind_raw_global(ch, p, b, h, t0);
  ch.L = L;
  float* small = reinterpret_cast<float*>(base + Lo::small);
  bind_small(ch, small);
  ch.Kr = reinterpret_cast<OpT*>(base + Lo::Kr);
  ch.Qr = reinterpret_cast<OpT*>(base + Lo::Qr);
  ch.Kc = reinterpret_cast<OpT*>(base + Lo::Kc);
  OpT* sTb = reinterpret_cast<OpT*>(base + Lo::Tb);
  OpT* sQb = reinterpret_cast<OpT*>(base + Lo::Qb);
  OpT* sXb = reinterpret_cast<OpT*>(base + Lo::Xb);
  OpT* sAb = reinterpret_cast<OpT*>(base + Lo::Ab);
  float* sA = reinterpret_cast<float*>(base + Lo::As);

  if constexpr (prep_staged<CF>()) {
    // raw rows by TMA (rows past T arrive as zeros); the operand build reads
    // them from shared memory
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + Lo::bar);
    if (threadIdx.x == 0) {
      mbar_init(bar, 1);
      fence_mbar_init();
      mbar_expect_tx(bar, (unsigned)(C * kKD * 8));
      tma_load_4d(base + Lo::raw_k, &maps.k, 0, h, t0, b, bar);
      tma_load_4d(base + Lo::raw_q, &maps.q, 0, h, t0, b, bar);
      tma_load_4d(base + Lo::raw_g, &maps.g, 0, h, t0, b, bar);
    }
    __syncthreads();  // the barrier's initialisation is visible before anyone waits on it
    Chunk<CF> src = ch;
    src.k = reinterpret_cast<const bf16*>(base + Lo::raw_k);
    src.q = reinterpret_cast<const bf16*>(base + Lo::raw_q);
    src.g = reinterpret_cast<const float*>(base + Lo::raw_g);
    src.ldr = kKD;
    prep_chunk<CF, kPrepThreads, false, true>(ch, &src, bar, p.status);
    __syncthreads();
    zero_upper_blocks<CF>(sQb);  // over the raw g rows, dead now
    zero_upper_blocks<CF>(sTb);
  } else {
    zero_upper_blocks<CF>(sQb);
    zero_upper_blocks<CF>(sTb);
    prep_chunk<CF, kPrepThreads>(ch);
    __syncthreads();
  }
  chunk_scores(ch, sA, sAb, sQb);
  chunk_solve<CF>(sA, sAb, sTb, sXb);

  // W0 = T Kr, written over Kr once every warp has read it
  {
    const int I = warp / NJ, n0 = (warp % NJ) * 8 * NTW;
    float acc[1][NTW][4];
    zero_acc(acc);
    wgemm<1, NTW, true, false>(acc, sTb, CF::LDC, ch.Kr, CF::LDK, 16 * I, n0, 0, 16 * (I + 1));
    __syncthreads();
    store_acc(ch.Kr, CF::LDK, acc, 16 * I, n0);
  }

  if constexpr (CF::F32) {
    // padded record, blocks as they lie in shared memory
    char* rec = static_cast<char*>(p.rec) + cc * R::bytes;
    const char* src[6] = {base + Lo::Qr, base + Lo::Kc, base + Lo::Kr, base + Lo::Tb, base + Lo::Qb,
                          reinterpret_cast<const char*>(ch.fr)};
    const size_t dst[6] = {R::Qr, R::Kc, R::W0, R::T, R::Q, R::F};
    const size_t len[6] = {R::Kc - R::Qr, R::W0 - R::Kc, R::T - R::W0, R::Q - R::T, R::F - R::Q, 3 * kKD * 4};
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 6; ++i)
      for (size_t o = (size_t)threadIdx.x * 16; o < len[i]; o += (size_t)blockDim.x * 16)
        *reinterpret_cast<int4*>(rec + dst[i] + o) = *reinterpret_cast<const int4*>(src[i] + o);
  } else {
    // swizzled tensor-core record with the scale factors folded in, assembled
    // in shared memory and written by bulk stores (one thread issues them)
    using RT = RecTc<CF>;
    char* rec = static_cast<char*>(p.rec) + cc * RT::bytes;
    char* st = base + Lo::St;
    __syncthreads();
    // Qs = scale fr Qr, Kf = fL Kc, Wf = fr W0, each rewritten swizzled over its
    // own padded tile (through registers): thread t owns keys 8(t%16)..+7 of
    // rows t/16, t/16 + 16, ...
    {
      constexpr int RPT = C / (kPrepThreads / 16);
      const int g = threadIdx.x & 15, r0 = threadIdx.x >> 4;
      char* tiles[3] = {base + Lo::Qr, base + Lo::Kc, base + Lo::Kr};
      uint4 v[3][RPT];
#pragma unroll
      for (int m = 0; m < 3; ++m) {
        const float* fac = m == 1 ? ch.fL : ch.fr;
        const float mul = m == 0 ? p.scale : 1.f;
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = mul * fac[8 * g + i];
#pragma unroll
        for (int j = 0; j < RPT; ++j) {
          float x[8];
          ld8(x, reinterpret_cast<const OpT*>(tiles[m]) + (r0 + 16 * j) * CF::LDK + 8 * g);
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] *= f[i];
          v[m][j] = pack8(x);
        }
      }
      __syncthreads();
#pragma unroll
      for (int m = 0; m < 3; ++m)
#pragma unroll
        for (int j = 0; j < RPT; ++j)
          *reinterpret_cast<uint4*>(tiles[m] + tc::sw_off(r0 + 16 * j, 8 * g, C)) = v[m][j];
    }
    // those three tiles and the factors leave while T, Qq, Qt are built
    fence_async_shared();
    __syncthreads();
    if (threadIdx.x == 0) {
      static_assert(RT::Kf == RT::Qs + (size_t)C * 256 && RT::Wf == RT::Kf + (size_t)C * 256, "record tile order");
      bulk_s2g(rec + RT::Qs, base + Lo::Qr, C * 256);
      bulk_s2g(rec + RT::Kf, base + Lo::Kc, C * 256);
      bulk_s2g(rec + RT::Wf, base + Lo::Kr, C * 256);
      bulk_s2g(rec + RT::F, ch.fr, 3 * kKD * 4);
      bulk_commit();
    }
    // T, Qq = scale Q: thread t owns columns 8(t%8)..+7 of rows t/8, t/8 + 32, ...
    // (columns >= C zero); Qt = scale Q^T: warp w owns output columns
    // 8(w%8)..+7 and lane l output row l, l + 32, ..., so the column reads of
    // the source are consecutive along a row (no bank conflicts)
    {
#pragma unroll 1
      for (int m = 0; m < 3; ++m) {
        char* dst = st + (size_t)m * C * 128;  // T, Qq, Qt: the record's order
        const float mul = m >= 1 ? p.scale : 1.f;
        const OpT* src = m == 0 ? sTb : sQb;
        const bool tr = m >= 2;
        const int g = tr ? (warp & 7) : (threadIdx.x & 7);
        const int r0 = tr ? (threadIdx.x & 31) + 32 * (warp >> 3) : threadIdx.x >> 3;
        const int rs = tr ? 32 * (kPrepThreads / 256) : kPrepThreads / 8;
        for (int r = r0; r < C; r += rs) {
          float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (8 * g < C) {
            if (!tr) {
              ld8(x, src + r * CF::LDC + 8 * g);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) x[i] = to_f(src[(8 * g + i) * CF::LDC + r]);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] *= mul;
          }
          *reinterpret_cast<uint4*>(dst + tc::sw_off(r, 8 * g, C)) = pack8(x);
        }
      }
    }
    fence_async_shared();
    __syncthreads();
    if (threadIdx.x == 0) {
      static_assert(RT::Qq == RT::T + (size_t)C * 128, "record tile order");
      bulk_s2g(rec + RT::T, st, 2 * C * 128);
      bulk_s2g(rec + RT::Qt, st + 2 * C * 128, C * 128);
      bulk_commit();
      bulk_wait_read<0>();  // shared memory stays valid until the stores have read it
    }
  }
}

template <class CF>
size_t prep_dbg_bytes() {
  return CF::F32 ? PrepLayout<CF>::bytes : 0;
}

template <class CF>
int launch_prep(const ScanParams& p, cudaStream_t st) {
  const size_t smem = CF::F32 ? 0 : PrepLayout<CF>::bytes;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(scan_prep_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return check_launch("cudaFuncSetAttribute(scan_prep_kernel)");
    configured = true;
  }
  PrepMaps maps;
  if constexpr (prep_staged<CF>()) {
    int rc = encode_bthd(&maps.q, p.q, true, p.B, p.T, p.H, kKD, kKD, CF::C, false);
    if (rc == KDN_OK) rc = encode_bthd(&maps.k, p.k, true, p.B, p.T, p.H, kKD, kKD, CF::C, false);
    if (rc == KDN_OK) rc = encode_bthd(&maps.g, p.g, false, p.B, p.T, p.H, kKD, kKD, CF::C, false);
    if (rc != KDN_OK) return rc;
  } else {
    memset(&maps, 0, sizeof(maps));
  }
  scan_prep_kernel<CF><<<dim3(p.c_hi - p.c_lo, p.B * p.H), kPrepThreads, smem, st>>>(p, maps);
  return check_launch("scan_prep_kernel");
}

template int launch_prep<Cfg<true, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_prep<Cfg<true, 64, float>>(const ScanParams&, cudaStream_t);
template int launch_prep<Cfg<false, 64, bf16>>(const ScanParams&, cudaStream_t);
template int launch_prep<Cfg<false, 32, float>>(const ScanParams&, cudaStream_t);
template size_t prep_dbg_bytes<Cfg<true, 64, float>>();
template size_t prep_dbg_bytes<Cfg<false, 32, float>>();

}  // namespace kdn
