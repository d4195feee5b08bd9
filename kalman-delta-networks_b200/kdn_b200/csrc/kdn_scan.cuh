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
constexpr int kSeqThreads = 512;  // sequential kernels: 16 warps

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
  // the bf16 diagonal scan runs 64-token chunks over a 32-local gate prefix:
  // the C ABI turns the prefix into a 64-local one first (and folds the gate
  // cotangent back), see kdn_scan_api.cu
  static_assert(C % CG == 0, "internal chunk must be a multiple of the boundary gate chunk");
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
  void* rec;  // [BH][NT] chunk records (Rec<CF>): Qr, Kc, W0, T, Q, gate factors
  void* h;    // [BH][NT][KD/BV][KD][LDV] OpT, chunk-start states scaled by fr
  void* dh;   // [BH][NT][KD/BV][KD][LDV] OpT, chunk-end state adjoints scaled by fL
  int* status;  // [flags, debug poll limit]: bounded waits set kStatusGaveUp / kStatusSlowWait in word 0
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
  // the launch covers chunks [c_lo, c_hi) of every stream (the C ABI passes
  // the whole sequence; a sequential pass over a sub-range starts from S0 /
  // dST and ends in ST / dS0 at the range's ends)
  int c_lo, c_hi;
  float scale;
  // state-map mode of the tensor-core sequential forward (sequence
  // parallelism): blockIdx.z = 0 carries initial_state with the values v to
  // ST, blockIdx.z = 1 carries the identity with zero values to ST2 (the
  // segment's linear state map); neither writes o or h
  int state_map;
  float* ST2;
  // packed variable-length batch (B = 1, NT = the global chunk count): the
  // chunk-parallel kernels take chunk c's tokens from the table, the
  // sequential ones run one (sequence, head) stream per CTA pair
  Varlen vl;
};

__host__ __device__ constexpr size_t A128(size_t x) { return align_up(x, 128); }
__host__ __device__ constexpr size_t cmax(size_t a, size_t b) { return a > b ? a : b; }

// Per-chunk record: written once by the chunk-parallel pass, read by the
// sequential passes (and T, Q by the chunk-parallel backward).  Rows are
// padded exactly like the shared-memory operands, so each block (or the
// whole record) moves with one bulk copy.
//   Qr, Kc, W0 = T Kr  [C][LDK] OpT;  T, Q [C][LDC] OpT;  fr, fL, 2^g_L [3][KD] fp32
template <class CF>
struct Rec {
  static constexpr size_t sz = sizeof(typename CF::OpT);
  static constexpr int C = CF::C;
  static constexpr size_t Qr = 0;
  static constexpr size_t Kc = Qr + (size_t)C * CF::LDK * sz;
  static constexpr size_t W0 = Kc + (size_t)C * CF::LDK * sz;
  static constexpr size_t T = W0 + (size_t)C * CF::LDK * sz;
  static constexpr size_t Q = T + (size_t)C * CF::LDC * sz;
  static constexpr size_t F = Q + (size_t)C * CF::LDC * sz;
  static constexpr size_t bytes = A128(F + 3 * kKD * 4);
  static_assert(Kc % 128 == 0 && T % 128 == 0 && F % 128 == 0, "16-byte aligned blocks");
};

// Tensor-core record (bf16 precision): tiles in the swizzled layout of
// kdn_tc.cuh, with the chunk's scale factors folded in so that the
// sequential passes carry the unscaled state:
//   T, Qq = scale Q, Qt = scale Q^T              [C][64] (columns >= C unused)
//   Qs = scale fr Qr,  Kf = fL Kc,  Wf = fr W0   [2][C][64] (64 keys per block)
//   fr, fL, 2^g_L                                  [3][KD] fp32
// The forward reads [0, fwd_end), the reverse sweep [bwd_begin, bytes).
template <class CF>
struct RecTc {
  static constexpr int C = CF::C;
  static constexpr size_t T = 0;
  static constexpr size_t Qq = T + (size_t)C * 128;
  static constexpr size_t Qs = Qq + (size_t)C * 128;
  static constexpr size_t Kf = Qs + (size_t)C * 256;
  static constexpr size_t Wf = Kf + (size_t)C * 256;
  static constexpr size_t F = Wf + (size_t)C * 256;
  static constexpr size_t Qt = F + align_up(3 * kKD * 4, 1024);
  static constexpr size_t bytes = Qt + (size_t)C * 128;
  static constexpr size_t fwd_end = Qt;
  static constexpr size_t bwd_begin = Qs;
  static_assert(bytes % 1024 == 0 && Qs % 1024 == 0, "1024-byte aligned tiles");
};
template <class CF>
using RecOf = typename std::conditional<CF::F32, Rec<CF>, RecTc<CF>>::type;

// One value tile of a chunk's state in shared memory (padded): [KD][LDV] OpT.
template <class CF>
__host__ __device__ constexpr size_t state_block_bytes() {
  return A128((size_t)kKD * CF::LDV * sizeof(typename CF::OpT));
}
// ... and in HBM (h, dh): the padded tile (fp32 precision, states scaled by
// fr / fL) or the swizzled bf16 tile [KD][64] of the unscaled state.
template <class CF>
__host__ __device__ constexpr size_t hblock_bytes() {
  return CF::F32 ? state_block_bytes<CF>() : (size_t)kKD * 64 * 2;
}

// Per-chunk views of the raw inputs (rows in shared memory or straight in
// HBM), the per-row / per-channel scalars and the gated operands.
template <class CF>
struct Chunk {
  using OpT = typename CF::OpT;
  // raw inputs: row i of q, k, g at ptr + i * ldr, of kappa at kap + i * ldk;
  // beta at beta[i * ldb]
  const bf16* q;
  const bf16* k;
  const float* g;
  const float* kap;   // diag
  const float* beta;  // iso
  int ldr, ldb, ldk;
  // per-row / per-channel scalars
  float* rq;  // iso rstd of q rows
  float* rk;  // iso rstd of k rows
  float* fr;
  float* fL;
  float* gL;
  float* gmid;   // gate at the reference row, per channel
  float* glast;  // gate at the last valid row, per channel
  float* red;    // [32] scratch
  float* rb;     // iso beta of the rows (0 past the chunk's end)
  // operands
  OpT* Kr;
  OpT* Qr;
  OpT* Kc;
  int L;
  int m;
  bool fast;
};

// Per-row / per-channel scalars of a chunk: rq, rk [C]; fr, fL, gL, gmid,
// glast [KD]; red [32].  fr, fL, gL are contiguous (the record's F block).
template <class CF>
__host__ __device__ constexpr size_t small_floats() {
  return 3 * CF::C + 5 * kKD + 32;
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
  ch.rb = ch.red + 32;
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

// First token and length of chunk c (a global chunk of a packed batch).
template <int C>
__device__ __forceinline__ void chunk_span(const ScanParams& p, int c, int& t0, int& L) {
  if (p.vl.on()) {  // (packed batches run the bf16 precision only: C = 64)
    int s;
    varlen_span(p.vl, c, t0, L, s);
  } else {
    t0 = c * C;
    L = min(C, p.T - t0);
  }
}

// Stream of a sequential-pass CTA (blockIdx.x): its chunk range, the row of
// the per-(b, h) records and states it reads, and its state index.  A packed
// batch runs its (sequence, head) streams longest sequence first.
struct SeqStream {
  int b, h, c_lo, c_hi;
  size_t rec_row;  // (b * H + h): chunk c's record is rec_row * NT + c
  size_t state;    // index of the [K][V] initial / final state
};
// CTAs (per value half) of a sequential pass: one per stream.
inline unsigned seq_streams(const ScanParams& p) {
  return (unsigned)(p.vl.on() ? (int64_t)p.vl.n * p.H : (int64_t)p.B * p.H);
}
__device__ __forceinline__ SeqStream seq_stream(const ScanParams& p, int slot) {
  SeqStream s;
  if (p.vl.on()) {
    const int seq = p.vl.order[slot / p.H];
    s.b = 0;
    s.h = slot - (slot / p.H) * p.H;
    s.c_lo = p.vl.chunk[seq];
    s.c_hi = p.vl.chunk[seq + 1];
    s.rec_row = (size_t)s.h;
    s.state = (size_t)seq * p.H + s.h;
  } else {
    s.b = slot / p.H;
    s.h = slot - s.b * p.H;
    s.c_lo = p.c_lo;
    s.c_hi = p.c_hi;
    s.rec_row = (size_t)slot;
    s.state = (size_t)slot;
  }
  return s;
}

// Zero rows [L, C) of a 128-byte-swizzled [C][64] bf16 tile (a packed
// batch's last chunk of a sequence: its TMA box runs into the next sequence).
template <int C>
__device__ __forceinline__ void zero_tail_rows(char* tile, int L, int tid, int nth) {
  for (int e = L * 8 + tid; e < C * 8; e += nth) {
    const int r = e >> 3, g = e & 7;  // row, 16-byte granule (swizzled by row % 8)
    *reinterpret_cast<uint4*>(tile + r * 128 + ((g ^ (r & 7)) << 4)) = make_uint4(0, 0, 0, 0);
  }
}

// Stage a chunk's q, k, g (and kappa or beta) rows in shared memory (cp.async,
// rows >= L zero-filled) and point the chunk view at them.
template <class CF>
__device__ __forceinline__ void load_raw(Chunk<CF>& ch, bf16* sq, bf16* sk, float* sg, float* skap,
                                         const ScanParams& p, int b, int h, int t0, int L) {
  constexpr bool SM = !CF::F32;
  const size_t r0 = tok_row(p, b, h, t0);
  const size_t rs = (size_t)p.H;
  copy_rows<SM>(sq, kKD * 2, p.q + r0 * kKD, rs * kKD * 2, CF::C, L, kKD * 2);
  copy_rows<SM>(sk, kKD * 2, p.k + r0 * kKD, rs * kKD * 2, CF::C, L, kKD * 2);
  copy_rows<SM>(sg, kKD * 4, p.g + r0 * kKD, rs * kKD * 4, CF::C, L, kKD * 4);
  if constexpr (CF::ISO) {
    for (int i = threadIdx.x; i < CF::C; i += blockDim.x) skap[i] = i < L ? p.beta[r0 + (size_t)i * rs] : 0.f;
  } else {
    copy_rows<SM>(skap, kKD * 4, p.kappa + r0 * kKD, rs * kKD * 4, CF::C, L, kKD * 4);
  }
  ch.q = sq;
  ch.k = sk;
  ch.g = sg;
  ch.kap = CF::ISO ? nullptr : skap;
  ch.beta = CF::ISO ? skap : nullptr;
  ch.ldr = kKD;
  ch.ldb = 1;
  ch.ldk = kKD;
}

// Point the chunk view at the rows in HBM.
template <class CF>
__device__ __forceinline__ void bind_raw_global(Chunk<CF>& ch, const ScanParams& p, int b, int h, int t0) {
  const size_t r0 = tok_row(p, b, h, t0);
  ch.q = p.q + r0 * kKD;
  ch.k = p.k + r0 * kKD;
  ch.g = p.g + r0 * kKD;
  ch.kap = CF::ISO ? nullptr : p.kappa + r0 * kKD;
  ch.beta = CF::ISO ? p.beta + r0 : nullptr;
  ch.ldr = p.H * kKD;
  ch.ldb = p.H;
  ch.ldk = p.H * kKD;
}

template <class CF>
__device__ __forceinline__ float kappa_at(const Chunk<CF>& ch, int i, int c) {
  if constexpr (CF::ISO) {
    return ch.beta[(size_t)i * ch.ldb] * ch.rk[i] * to_f(ch.k[(size_t)i * ch.ldr + c]);
  } else {
    return ch.kap[(size_t)i * ch.ldr + c];
  }
}
template <class CF>
__device__ __forceinline__ float khat_at(const Chunk<CF>& ch, int i, int c) {
  if constexpr (CF::ISO) {
    return ch.rk[i] * to_f(ch.k[(size_t)i * ch.ldr + c]);
  } else {
    return to_f(ch.k[(size_t)i * ch.ldr + c]);
  }
}
template <class CF>
__device__ __forceinline__ float qhat_at(const Chunk<CF>& ch, int i, int c) {
  if constexpr (CF::ISO) {
    return ch.rq[i] * to_f(ch.q[(size_t)i * ch.ldr + c]);
  } else {
    return to_f(ch.q[(size_t)i * ch.ldr + c]);
  }
}

// One row's raw values for the 8 channels a thread handles.
// k and q stay packed (8 bf16 in 16 bytes) until used, so that all of a
// thread's rows can be in flight at once.
template <class CF>
struct RawRow {
  float g[8], kap[CF::ISO ? 1 : 8];
  uint4 kp, qp;
  float beta;
};

__device__ __forceinline__ uint4 pack8(const float (&x)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
  return u;
}

__device__ __forceinline__ void unpack8(float (&d)[8], const uint4& u) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    d[2 * i] = f.x;
    d[2 * i + 1] = f.y;
  }
}

template <class CF>
__device__ __forceinline__ void load_row(RawRow<CF>& x, const Chunk<CF>& ch, int r, int c0) {
  if (r < ch.L) {
    const size_t o = (size_t)r * ch.ldr + c0;
    ld8(x.g, ch.g + o);
    x.kp = *reinterpret_cast<const uint4*>(ch.k + o);
    x.qp = *reinterpret_cast<const uint4*>(ch.q + o);
    if constexpr (CF::ISO) {
      x.beta = ch.beta[(size_t)r * ch.ldb];
    } else {
      ld8(x.kap, ch.kap + (size_t)r * ch.ldk + c0);
      x.beta = 1.f;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x.g[i] = 0.f;
      if constexpr (!CF::ISO) x.kap[i] = 0.f;
    }
    x.kp = x.qp = make_uint4(0, 0, 0, 0);
    x.beta = 0.f;
  }
}

// Gated operands of one row: Kr = k_hat 2^(g - rr), Qr = q_hat 2^(g - rr),
// Kc = kappa 2^(rc - g); zero rows past the chunk's end.  make_operands
// leaves them as 8 rounded OpT values per operand (bf16 precision: one 16-byte
// word each); store_operands writes them, SW: into 64-row swizzled
// tensor-core tiles instead of padded rows.
template <class CF>
__device__ __forceinline__ void make_operands(const Chunk<CF>& ch, int r, const RawRow<CF>& x, const float (&rr)[8],
                                              const float (&rc)[8], float qs, float ks, float (&kr)[8],
                                              float (&qr)[8], float (&kc)[8]) {
  if (r < ch.L) {
    const float bs = CF::ISO ? x.beta * ks : 1.f;
    float k8[8], q8[8];
    unpack8(k8, x.kp);
    unpack8(q8, x.qp);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float er = ex2a(x.g[i] - rr[i]);
      const float ec = ex2a(rc[i] - x.g[i]);
      kr[i] = k8[i] * ks * er;
      qr[i] = q8[i] * qs * er;
      kc[i] = (CF::ISO ? k8[i] : x.kap[i]) * bs * ec;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) kr[i] = qr[i] = kc[i] = 0.f;
  }
}
template <class CF, bool SW>
__device__ __forceinline__ void store_operands(const Chunk<CF>& ch, int r, int c0, const float (&kr)[8],
                                               const float (&qr)[8], const float (&kc)[8]) {
  if constexpr (SW) {
    // byte offset of (r, c0) in a [2][64][64] swizzled tile
    const uint32_t o = (uint32_t)((c0 >> 6) * 64 * 128 + r * 128 + ((((c0 & 63) >> 3) ^ (r & 7)) << 4));
    st8(reinterpret_cast<typename CF::OpT*>(reinterpret_cast<char*>(ch.Kr) + o), kr);
    st8(reinterpret_cast<typename CF::OpT*>(reinterpret_cast<char*>(ch.Qr) + o), qr);
    st8(reinterpret_cast<typename CF::OpT*>(reinterpret_cast<char*>(ch.Kc) + o), kc);
  } else {
    st8(ch.Kr + r * CF::LDK + c0, kr);
    st8(ch.Qr + r * CF::LDK + c0, qr);
    st8(ch.Kc + r * CF::LDK + c0, kc);
  }
}
template <class CF, bool SW = false>
__device__ __forceinline__ void build_operands(const Chunk<CF>& ch, int r, int c0, const RawRow<CF>& x,
                                               const float (&rr)[8], const float (&rc)[8], float qs, float ks) {
  float kr[8], qr[8], kc[8];
  make_operands(ch, r, x, rr, rc, qs, ks, kr, qr, kc);
  store_operands<CF, SW>(ch, r, c0, kr, qr, kc);
}

// Row norms (iso), range check, per-channel factors and the three gated
// operands, for a block of NTH threads.  Thread t handles channels
// 8*(t%16) .. +7 of rows t/16, t/16 + NTH/16, ...; the 16 threads of a row
// are one half-warp, so row norms are half-warp shuffles.  All of a thread's
// rows (up to 4) are loaded ahead of their arithmetic (they may come straight
// from HBM).
// The operands are built with the fast-path reference (the gate of the
// middle row, known up front) and built again only when the range check
// sends the chunk to the exact path.  Contains one barrier (two when staged);
// the caller places the barrier that publishes the results.
// STAGED: the first build reads the q, k, g rows from shared-memory copies
// (`src`, rows of kKD, complete once `staged_bar` completes its first phase;
// beta and kappa stay where `src` points) that lie under the operand tiles it
// writes, so every thread builds all of its rows into registers before a
// barrier and stores them after it; the exact-path rebuild reads `ch` (the
// rows in HBM).
template <class CF, int NTH, bool SW = false, bool STAGED = false>
__device__ void prep_chunk(Chunk<CF>& ch, const Chunk<CF>* src = nullptr, uint64_t* staged_bar = nullptr,
                           int* status = nullptr) {
  constexpr int C = CF::C, RSTEP = NTH / 16, RPT = C / RSTEP, BATCH = RPT <= 4 ? RPT : 2;
  static_assert(NTH % 32 == 0 && C % RSTEP == 0 && RPT % BATCH == 0, "rows per thread");
  const Chunk<CF>& in = STAGED ? *src : ch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = ch.L;
  ch.m = L >= C ? C / 2 : (((L - 1) / 2) & ~15);
  const int c0 = (threadIdx.x & 15) * 8, rt = threadIdx.x >> 4;
  // staged: the rows still in HBM (iso beta, diag kappa) are requested before
  // the wait for the staged ones, so that both latencies overlap
  float pb[STAGED && CF::ISO ? RPT : 1], pk[STAGED && !CF::ISO ? RPT : 1][8];
  if constexpr (STAGED) {
#pragma unroll
    for (int j = 0; j < RPT; ++j) {
      const int r = rt + j * RSTEP;
      if constexpr (CF::ISO) {
        pb[j] = r < L ? in.beta[(size_t)r * in.ldb] : 0.f;
      } else {
        if (r < L) {
          ld8(pk[j], in.kap + (size_t)r * in.ldk + c0);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) pk[j][i] = 0.f;
        }
      }
    }
    mbar_wait(staged_bar, 0, status);
  }
  float gm[8], gl[8];
  ld8(gm, in.g + (size_t)ch.m * in.ldr + c0);
  ld8(gl, in.g + (size_t)(L - 1) * in.ldr + c0);
  float rng = 0.f;
  // iso: row scales 1/|q|, 1/|k| (half-warp sums), kept with beta per row
  auto row_scales = [&](const RawRow<CF>& x, int r, float& qs, float& ks) {
    qs = ks = 1.f;
    if constexpr (CF::ISO) {
      float sq = 0.f, sk = 0.f, k8[8], q8[8];
      unpack8(k8, x.kp);
      unpack8(q8, x.qp);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sq = fmaf(q8[i], q8[i], sq);
        sk = fmaf(k8[i], k8[i], sk);
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
      }
      qs = rsqrtf(sq + 1e-6f);
      ks = rsqrtf(sk + 1e-6f);
      if ((threadIdx.x & 15) == 0) {
        ch.rq[r] = qs;
        ch.rk[r] = ks;
        ch.rb[r] = x.beta;
      }
    }
    if (r < L) {
#pragma unroll
      for (int i = 0; i < 8; ++i) rng = fmaxf(rng, fabsf(x.g[i] - gm[i]));
    }
  };
  if constexpr (STAGED) {
    // row by row from shared memory into rounded operand words; the stores
    // wait for every thread's reads
    static_assert(!CF::F32, "staged build: bf16 operands");
    uint4 okr[RPT], oqr[RPT], okc[RPT];
#pragma unroll
    for (int j = 0; j < RPT; ++j) {
      const int r = rt + j * RSTEP;
      RawRow<CF> x;
      if (r < L) {
        const size_t o = (size_t)r * in.ldr + c0;
        ld8(x.g, in.g + o);
        x.kp = *reinterpret_cast<const uint4*>(in.k + o);
        x.qp = *reinterpret_cast<const uint4*>(in.q + o);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x.g[i] = 0.f;
        x.kp = x.qp = make_uint4(0, 0, 0, 0);
      }
      if constexpr (CF::ISO) {
        x.beta = pb[j];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x.kap[i] = pk[j][i];
        x.beta = 1.f;
      }
      float qs, ks, kr[8], qr[8], kc[8];
      row_scales(x, r, qs, ks);
      make_operands(ch, r, x, gm, gm, qs, ks, kr, qr, kc);
      okr[j] = pack8(kr);
      oqr[j] = pack8(qr);
      if constexpr (!SW) {
        // chunk prep (padded tiles): no raw row is staged under Kc, so Kc is
        // stored now and only Kr, Qr wait for the barrier (16 registers fewer;
        // the kernel spilled at its 128-register cap when all three waited)
        st8(ch.Kc + r * CF::LDK + c0, kc);
      } else {
        okc[j] = pack8(kc);
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < RPT; ++j) {
      const int r = rt + j * RSTEP;
      float kr[8], qr[8], kc[8];
      unpack8(kr, okr[j]);
      unpack8(qr, oqr[j]);
      if constexpr (!SW) {
        st8(ch.Kr + r * CF::LDK + c0, kr);
        st8(ch.Qr + r * CF::LDK + c0, qr);
      } else {
        unpack8(kc, okc[j]);
        store_operands<CF, SW>(ch, r, c0, kr, qr, kc);
      }
    }
  } else {
#pragma unroll
    for (int j0 = 0; j0 < RPT; j0 += BATCH) {
      RawRow<CF> x[BATCH];
#pragma unroll
      for (int j = 0; j < BATCH; ++j) load_row(x[j], in, rt + (j0 + j) * RSTEP, c0);
#pragma unroll
      for (int j = 0; j < BATCH; ++j) {
        const int r = rt + (j0 + j) * RSTEP;
        float qs, ks;
        row_scales(x[j], r, qs, ks);
        build_operands<CF, SW>(ch, r, c0, x[j], gm, gm, qs, ks);
      }
    }
  }
  rng = warp_max(rng);
  if (lane == 0) ch.red[warp] = rng;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < NTH / 32; ++w) tot = fmaxf(tot, ch.red[w]);
  ch.fast = tot <= kRngMax;
  float rr[8], rc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    rr[i] = ch.fast ? gm[i] : 0.f;
    rc[i] = ch.fast ? gm[i] : gl[i];
  }
  if (threadIdx.x < 16) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ch.fr[c0 + i] = ex2(rr[i]);
      ch.fL[c0 + i] = ex2(gl[i] - rc[i]);
      ch.gL[c0 + i] = ex2(gl[i]);
      ch.gmid[c0 + i] = gm[i];
      ch.glast[c0 + i] = gl[i];
    }
  }
  if (!ch.fast) {
#pragma unroll 1
    for (int j = 0; j < RPT; ++j) {
      const int r = rt + j * RSTEP;
      RawRow<CF> x;
      load_row(x, ch, r, c0);
      const float qs = CF::ISO ? ch.rq[r] : 1.f, ks = CF::ISO ? ch.rk[r] : 1.f;
      build_operands<CF, SW>(ch, r, c0, x, rr, rc, qs, ks);
    }
  }
}

// Strictly lower A (fp32 sA for the diagonal-block inversion, OpT sAb for
// the tensor-core merges) and lower Q (OpT sQ).  Blocks above the diagonal
// are never written: the callers zero them once.  Ends with a barrier.
template <class CF>
__device__ void chunk_scores(const Chunk<CF>& ch, float* sA, typename CF::OpT* sAb, typename CF::OpT* sQ) {
  constexpr int C = CF::C, NB = CF::NB;
  using OpT = typename CF::OpT;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (ch.fast) {
    constexpr int ntri = NB * (NB + 1) / 2;
    for (int job = warp; job < ntri; job += nw) {
      int J = job, I = 0;
      while (J > I) {
        J -= I + 1;
        ++I;
      }
      float acc[2][2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[i][n][e] = 0.f;
      wgemm_dual<2, true, true>(acc, ch.Kr, ch.Qr, CF::LDK, ch.Kc, CF::LDK, 16 * I, 16 * J, 0, kKD);
      const int lane = threadIdx.x & 31;
      const int g = lane >> 2, t = lane & 3;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = 16 * I + g + 8 * h, j = 16 * J + nt * 8 + 2 * t;
          const float a0 = j < i ? acc[0][nt][2 * h] : 0.f, a1 = j + 1 < i ? acc[0][nt][2 * h + 1] : 0.f;
          const float q0 = j <= i ? acc[1][nt][2 * h] : 0.f, q1 = j + 1 <= i ? acc[1][nt][2 * h + 1] : 0.f;
          st_pair(sA + i * CF::LDA + j, a0, a1);
          st_pair(sAb + i * CF::LDC + j, a0, a1);
          st_pair(sQ + i * CF::LDC + j, q0, q1);
        }
    }
  } else {
    // exact: 2^(g_i - g_j) <= 1 evaluated per element
    for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
      const int i = e / C, j = e - i * C;
      if ((j >> 4) > (i >> 4)) continue;
      float a = 0.f, qq = 0.f;
      if (j <= i && i < ch.L) {
        for (int c = 0; c < kKD; ++c) {
          const float f = kappa_at(ch, j, c) * ex2(ch.g[(size_t)i * ch.ldr + c] - ch.g[(size_t)j * ch.ldr + c]);
          a = fmaf(khat_at(ch, i, c), f, a);
          qq = fmaf(qhat_at(ch, i, c), f, qq);
        }
      }
      a = j < i ? a : 0.f;
      sA[i * CF::LDA + j] = a;
      sAb[i * CF::LDC + j] = from_f<OpT>(a);
      sQ[i * CF::LDC + j] = from_f<OpT>(qq);
    }
  }
  __syncthreads();
}

// Zero the blocks above the 16x16 block diagonal of a C x C OpT buffer.
template <class CF>
__device__ __forceinline__ void zero_upper_blocks(typename CF::OpT* M) {
  constexpr int C = CF::C;
  for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
    const int i = e / C, j = e - i * C;
    if ((j >> 4) > (i >> 4)) M[i * CF::LDC + j] = from_f<typename CF::OpT>(0.f);
  }
}

// T = (I + A)^-1 for strictly lower A: 16x16 diagonal blocks by forward
// substitution (fp32, one lane per column), then recursive doubling on the
// tensor cores, T21 = -T22 (A21 T11), first for 16-row pairs, then for the
// 32-row halves.  Writes the OpT sTb (upper blocks must be zero already);
// sXb is OpT scratch of the same shape.  Ends with a barrier.
template <class CF>
__device__ void chunk_solve(const float* sA, const typename CF::OpT* sAb, typename CF::OpT* sTb,
                            typename CF::OpT* sXb) {
  constexpr int NB = CF::NB, LDA = CF::LDA, LDC = CF::LDC;
  using OpT = typename CF::OpT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < NB && lane < 16) {
    // column j of the block's inverse, right-looking: once col[l] is final it
    // updates every later row, so consecutive updates are independent (the
    // terms still accumulate in ascending l, and col[l] = 0 for l < j)
    const int o = warp * 16, j = lane;
    float col[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) col[i] = (i == j) ? 1.f : 0.f;
#pragma unroll
    for (int l = 0; l < 15; ++l)
#pragma unroll
      for (int i = l + 1; i < 16; ++i) col[i] = fmaf(-sA[(o + i) * LDA + o + l], col[l], col[i]);
#pragma unroll
    for (int i = 0; i < 16; ++i) sTb[(o + i) * LDC + o + j] = from_f<OpT>(col[i]);
  }
  __syncthreads();
  // pairs of 16-row blocks
  if (warp < NB / 2) {
    const int b0 = 32 * warp, b1 = b0 + 16;
    float acc[1][2][4];
    zero_acc(acc);
    wgemm<1, 2, true, false>(acc, sAb, LDC, sTb, LDC, b1, b0, b0, b1);
    store_acc(sXb, LDC, acc, b1, b0);
  }
  __syncthreads();
  if (warp < NB / 2) {
    const int b0 = 32 * warp, b1 = b0 + 16;
    float acc[1][2][4];
    zero_acc(acc);
    wgemm<1, 2, true, false>(acc, sTb, LDC, sXb, LDC, b1, b0, b1, b1 + 16);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[0][nt][e] = -acc[0][nt][e];
    store_acc(sTb, LDC, acc, b1, b0);
  }
  __syncthreads();
  if constexpr (NB == 4) {
    // 32-row halves: T[32:64, 0:32] = -T[32:64, 32:64] (A[32:64, 0:32] T[0:32, 0:32])
    const int I = 2 + (warp >> 1), J = warp & 1;
    if (warp < 4) {
      float acc[1][2][4];
      zero_acc(acc);
      wgemm<1, 2, true, false>(acc, sAb, LDC, sTb, LDC, 16 * I, 16 * J, 16 * J, 32);
      store_acc(sXb, LDC, acc, 16 * I, 16 * J);
    }
    __syncthreads();
    if (warp < 4) {
      float acc[1][2][4];
      zero_acc(acc);
      wgemm<1, 2, true, false>(acc, sTb, LDC, sXb, LDC, 16 * I, 16 * J, 32, 16 * (I + 1));
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[0][nt][e] = -acc[0][nt][e];
      store_acc(sTb, LDC, acc, 16 * I, 16 * J);
    }
    __syncthreads();
  }
  static_assert(NB == 2 || NB == 4, "chunk of 32 or 64 tokens");
}

// Contiguous copy of `bytes` (a multiple of 16) by the whole block:
// cp.async towards shared memory, or plain 16-byte copies in the fp32 debug
// precision (where both sides are global memory).
template <class CF>
__device__ __forceinline__ void copy_block(void* dst, const void* src, size_t bytes) {
  char* d = static_cast<char*>(dst);
  const char* s = static_cast<const char*>(src);
  for (size_t o = (size_t)threadIdx.x * 16; o < bytes; o += (size_t)blockDim.x * 16) {
    if constexpr (CF::F32) {
      *reinterpret_cast<int4*>(d + o) = *reinterpret_cast<const int4*>(s + o);
    } else {
      cp_async16(d + o, s + o);
    }
  }
}

}  // namespace kdn
