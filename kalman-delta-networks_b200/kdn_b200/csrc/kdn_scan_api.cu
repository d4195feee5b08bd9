// C ABI of the chunked memory scan: argument validation, caller-owned saved
// state and workspace layout, and dispatch to the kernel instantiations.
#include <math.h>
#include <stdlib.h>

#include "kdn_scan.cuh"

namespace kdn {

template <class CF> int launch_fwd(const ScanParams&, cudaStream_t);
template <class CF> int launch_bwd(const ScanParams&, cudaStream_t);
template <class CF> int launch_prep(const ScanParams&, cudaStream_t);
template <class CF> int launch_fwd_seq(const ScanParams&, cudaStream_t);
template <class CF> int launch_bwd_state(const ScanParams&, cudaStream_t);
template <class CF> size_t prep_dbg_bytes();
template <class CF> size_t fwd_dbg_bytes();
template <class CF> size_t state_bytes();
template <class CF> size_t chunk_bytes();

using IsoB = Cfg<true, 64, bf16>;
using IsoF = Cfg<true, 64, float>;
using DiagB = Cfg<false, 64, bf16>;
using DiagF = Cfg<false, 32, float>;

namespace {

// saved     = [status word | chunk records | chunk-start states h | 64-local gate prefix (bf16 diag)]
// workspace = [status word | chunk-end adjoints dh | fp32-precision scratch]
constexpr size_t kHeader = 256;
constexpr int kVT = kVD / kBV;

struct Sizes {
  int64_t C, NT, BH;
  size_t rec, h, dh;
  size_t g64;  // bf16 diagonal scan: the gate prefix restarted every 64 tokens
  size_t fwd_stride, bwd_stride;  // per-CTA scratch of the fp32 precision
  size_t dbg_fwd, dbg_bwd;
};

template <class CF>
void layout_sizes(Sizes* s) {
  s->rec = align_up(RecOf<CF>::bytes * s->BH * s->NT, 256);
  s->h = align_up(hblock_bytes<CF>() * kVT * s->BH * s->NT, 256);
  s->dh = s->h;
}

bool sizes_of(const KdnScanArgs* a, Sizes* s) {
  if (!a || (a->variant != KDN_ISO && a->variant != KDN_DIAG) ||
      (a->precision != KDN_PREC_BF16 && a->precision != KDN_PREC_FP32))
    return false;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->K != kKD || a->V != kVD) return false;
  const bool iso = a->variant == KDN_ISO, f32 = a->precision == KDN_PREC_FP32;
  // the bf16 kernels run 64-token chunks for both variants; the fp32 debug
  // build of the diagonal scan keeps the boundary's 32-token chunks
  s->C = (iso || !f32) ? 64 : 32;
  s->NT = (a->T + s->C - 1) / s->C;
  s->BH = a->B * a->H;
  if (a->num_seqs > 0) {
    // packed batch: the sequences' own chunks, numbered globally (B = 1, bf16)
    if (!a->varlen_table || a->B != 1 || f32 || a->num_chunks < a->num_seqs || a->num_chunks * 64 < a->T ||
        a->num_chunks > a->T)
      return false;
    s->NT = a->num_chunks;
  }
  if (iso) {
    f32 ? layout_sizes<IsoF>(s) : layout_sizes<IsoB>(s);
  } else {
    f32 ? layout_sizes<DiagF>(s) : layout_sizes<DiagB>(s);
  }
  s->fwd_stride = s->bwd_stride = s->dbg_fwd = s->dbg_bwd = 0;
  s->g64 = (!iso && !f32) ? align_up((size_t)4 * a->B * a->T * a->H * a->K, 256) : 0;
  if (f32) {
    const size_t pr = iso ? prep_dbg_bytes<IsoF>() : prep_dbg_bytes<DiagF>();
    const size_t f = iso ? fwd_dbg_bytes<IsoF>() : fwd_dbg_bytes<DiagF>();
    const size_t st = iso ? state_bytes<IsoF>() : state_bytes<DiagF>();
    const size_t ck = iso ? chunk_bytes<IsoF>() : chunk_bytes<DiagF>();
    // the two kernels of each direction index per-CTA slices with one stride
    const size_t ctas = (size_t)(s->NT > kVT ? s->NT : kVT) * s->BH;
    s->fwd_stride = pr > f ? pr : f;
    s->bwd_stride = st > ck ? st : ck;
    s->dbg_fwd = align_up(s->fwd_stride * ctas, 256);
    s->dbg_bwd = align_up(s->bwd_stride * ctas, 256);
  }
  return true;
}

int fill_params(const KdnScanArgs* a, const Sizes& s, ScanParams* p) {
  if (!(isfinite(a->scale))) return set_error(KDN_ERR_INVALID, "kdn_scan: scale must be finite");
  if (a->T > (1ll << 30) || s.BH > 65535 || s.NT > 2147483647ll / 64)
    return set_error(KDN_ERR_INVALID, "kdn_scan: size too large");
  *p = ScanParams{};
  p->q = static_cast<const bf16*>(a->q);
  p->k = static_cast<const bf16*>(a->k);
  p->v = static_cast<const bf16*>(a->v);
  p->g = a->g;
  p->beta = a->beta;
  p->kappa = a->kappa;
  p->S0 = a->initial_state;
  p->o = a->o;
  p->ST = a->final_state;
  char* sv = static_cast<char*>(a->saved);
  p->status = reinterpret_cast<int*>(sv);
  p->rec = sv + kHeader;
  p->h = sv + kHeader + s.rec;
  p->dO = a->dO;
  p->dST = a->d_final_state;
  p->dS0 = a->d_initial_state;
  p->dq = static_cast<bf16*>(a->dq);
  p->dk = static_cast<bf16*>(a->dk);
  p->dv = static_cast<bf16*>(a->dv);
  p->dg = a->dg;
  p->dbeta = a->dbeta;
  p->dkappa = a->dkappa;
  p->B = (int)a->B;
  p->T = (int)a->T;
  p->H = (int)a->H;
  p->NT = (int)s.NT;
  p->c_lo = 0;
  p->c_hi = (int)s.NT;
  p->scale = a->scale;
  p->vl = varlen_view(a->varlen_table, a->num_seqs);
  return KDN_OK;
}

// The diagonal scan's boundary gate prefix g restarts every 32 tokens; the
// bf16 kernels use 64-token chunks, whose prefix restarts every 64 tokens:
// g64[t] = g[t] + (t mod 64 >= 32 ? g[31 of the block] : 0).  One float4 of
// [B, T, H, K] per thread and step.
__global__ void gate_to64_kernel(const float4* __restrict__ g, float4* __restrict__ g64, int64_t T, int64_t HK4,
                                 int64_t n4) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n4; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / HK4, col = e - row * HK4, t = row % T, tb = t & 63;
    float4 x = g[e];
    if (tb >= 32) {
      const float4 y = g[(row - tb + 31) * HK4 + col];
      x.x += y.x;
      x.y += y.y;
      x.z += y.z;
      x.w += y.w;
    }
    g64[e] = x;
  }
}

// The cotangent of the 64-local prefix back to the boundary's 32-local one:
// rows 32..63 of a 64-token block also depend on row 31, which collects their
// cotangent.  One float4 column of one block per thread.
__global__ void gate_fold_kernel(float4* __restrict__ dg, int64_t T, int64_t HK4, int64_t NB64, int64_t n) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t col = e % HK4, bb = e / HK4, b = bb / NB64, blk = bb - b * NB64;
    const int64_t t31 = blk * 64 + 31, tend = t31 + 33 < T ? t31 + 33 : T;
    if (t31 + 1 >= tend) continue;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t t = t31 + 1; t < tend; ++t) {
      const float4 y = dg[(b * T + t) * HK4 + col];
      acc.x += y.x;
      acc.y += y.y;
      acc.z += y.z;
      acc.w += y.w;
    }
    float4& z = dg[(b * T + t31) * HK4 + col];
    z.x += acc.x;
    z.y += acc.y;
    z.z += acc.z;
    z.w += acc.w;
  }
}

// The same two conversions for a packed batch, whose 64-token chunks start
// at each sequence's first token (global chunk gc: tokens t0 .. t0 + L).
__global__ void gate_to64_varlen_kernel(const float4* __restrict__ g, float4* __restrict__ g64, Varlen v,
                                        int64_t HK4, int64_t n4) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n4; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t per = 64 * HK4, gc = e / per, rem = e - gc * per, r = rem / HK4, col = rem - r * HK4;
    int t0, L, sq;
    varlen_span(v, (int)gc, t0, L, sq);
    if (r >= L) continue;
    float4 x = g[(t0 + r) * HK4 + col];
    if (r >= 32) {
      const float4 y = g[(t0 + 31) * HK4 + col];
      x.x += y.x;
      x.y += y.y;
      x.z += y.z;
      x.w += y.w;
    }
    g64[(t0 + r) * HK4 + col] = x;
  }
}

__global__ void gate_fold_varlen_kernel(float4* __restrict__ dg, Varlen v, int64_t HK4, int64_t n) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t gc = e / HK4, col = e - gc * HK4;
    int t0, L, sq;
    varlen_span(v, (int)gc, t0, L, sq);
    if (L <= 32) continue;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 32; r < L; ++r) {
      const float4 y = dg[(t0 + r) * HK4 + col];
      acc.x += y.x;
      acc.y += y.y;
      acc.z += y.z;
      acc.w += y.w;
    }
    float4& z = dg[(t0 + 31) * HK4 + col];
    z.x += acc.x;
    z.y += acc.y;
    z.z += acc.z;
    z.w += acc.w;
  }
}

unsigned grid_for(int64_t n) {
  const int64_t blocks = (n + 255) / 256;
  return (unsigned)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

__global__ void status_init_kernel(int* status, int slow_polls) {
  status[0] = 0;
  status[1] = slow_polls;
}

// Clear the call's status header: word 0 collects the bounded waits' flags,
// word 1 is the debug poll limit of mbar_wait (KDN_B200_DEBUG_POLL_LIMIT,
// 0 or unset = off; a test sets it to make the slow-wait flag fire).
int reset_status(int* status, cudaStream_t st, const char* what) {
  const char* env = getenv("KDN_B200_DEBUG_POLL_LIMIT");
  const int slow = env ? atoi(env) : 0;
  if (slow <= 0) {
    if (cudaMemsetAsync(status, 0, 2 * sizeof(int), st) != cudaSuccess) return check_launch(what);
    return KDN_OK;
  }
  status_init_kernel<<<1, 1, 0, st>>>(status, slow);
  return check_launch(what);
}

}  // namespace
}  // namespace kdn

using namespace kdn;

extern "C" {

size_t kdn_scan_saved_bytes(const KdnScanArgs* a) {
  Sizes s;
  if (!sizes_of(a, &s)) return 0;
  return kHeader + s.rec + s.h + s.g64;
}

size_t kdn_scan_workspace_bytes(const KdnScanArgs* a) {
  Sizes s;
  if (!sizes_of(a, &s)) return 0;
  const size_t bwd = kHeader + s.dh + s.dbg_bwd;
  return bwd > s.dbg_fwd ? bwd : s.dbg_fwd;
}

int kdn_scan_fwd(const KdnScanArgs* a, kdn_stream_t stream) {
  Sizes s;
  if (!sizes_of(a, &s))
    return set_error(KDN_ERR_INVALID,
                     "kdn_scan_fwd: unsupported variant/precision or shape (K and V must be 128; a packed batch "
                     "needs B = 1, the bf16 precision and its kdn_varlen_plan table)");
  const int mode = a->mode;
  if (mode != KDN_SCAN_FULL && mode != KDN_SCAN_FWD_RECORDS && mode != KDN_SCAN_FWD_SEQUENTIAL &&
      mode != KDN_SCAN_FWD_STATE_MAP)
    return set_error(KDN_ERR_INVALID, "kdn_scan_fwd: mode %d is not a forward mode", mode);
  if (mode != KDN_SCAN_FULL && a->precision != KDN_PREC_BF16)
    return set_error(KDN_ERR_INVALID, "kdn_scan_fwd: the partial-pass modes need the bf16 precision");
  if (a->num_seqs > 0 && mode != KDN_SCAN_FULL)
    return set_error(KDN_ERR_INVALID, "kdn_scan_fwd: a packed batch runs mode 0 only");
  const bool need_o = mode == KDN_SCAN_FULL || mode == KDN_SCAN_FWD_SEQUENTIAL;
  if (!a->q || !a->k || !a->v || !a->g || (need_o && !a->o) || !a->saved ||
      (a->variant == KDN_ISO ? !a->beta : !a->kappa))
    return set_error(KDN_ERR_INVALID, "kdn_scan_fwd: null input/output pointer");
  if (mode == KDN_SCAN_FWD_STATE_MAP && (!a->final_state || !a->final_state_map))
    return set_error(KDN_ERR_INVALID, "kdn_scan_fwd: the state-map mode writes final_state and final_state_map");
  if (s.dbg_fwd && (!a->workspace || a->workspace_bytes < s.dbg_fwd))
    return set_error(KDN_ERR_WORKSPACE, "kdn_scan_fwd: workspace too small");
  ScanParams p;
  int rc = fill_params(a, s, &p);
  if (rc != KDN_OK) return rc;
  const cudaStream_t st = (cudaStream_t)stream;
  if (reset_status(p.status, st, "kdn_scan_fwd: status reset") != KDN_OK) return KDN_ERR_CUDA;
  p.dbg = static_cast<char*>(a->workspace);
  p.dbg_stride = s.fwd_stride;
  const bool iso = a->variant == KDN_ISO;
  if (a->precision == KDN_PREC_FP32) return iso ? launch_fwd<IsoF>(p, st) : launch_fwd<DiagF>(p, st);
  float* g64 = reinterpret_cast<float*>(static_cast<char*>(a->saved) + kHeader + s.rec + s.h);
  if (!iso && (mode == KDN_SCAN_FULL || mode == KDN_SCAN_FWD_RECORDS)) {
    // 32-local gate prefix -> 64-local, kept in `saved` for the later passes
    const int64_t HK4 = a->H * a->K / 4, n4 = a->B * a->T * HK4;
    if (p.vl.on()) {
      const int64_t nv = s.NT * 64 * HK4;
      gate_to64_varlen_kernel<<<grid_for(nv), 256, 0, st>>>(reinterpret_cast<const float4*>(a->g),
                                                            reinterpret_cast<float4*>(g64), p.vl, HK4, nv);
    } else {
      gate_to64_kernel<<<grid_for(n4), 256, 0, st>>>(reinterpret_cast<const float4*>(a->g),
                                                     reinterpret_cast<float4*>(g64), a->T, HK4, n4);
    }
    rc = check_launch("gate_to64_kernel");
    if (rc != KDN_OK) return rc;
  }
  if (!iso) p.g = g64;
  if (mode == KDN_SCAN_FULL) return iso ? launch_fwd<IsoB>(p, st) : launch_fwd<DiagB>(p, st);
  if (mode == KDN_SCAN_FWD_RECORDS) return iso ? launch_prep<IsoB>(p, st) : launch_prep<DiagB>(p, st);
  if (mode == KDN_SCAN_FWD_STATE_MAP) {
    p.state_map = 1;
    p.ST2 = a->final_state_map;
    p.o = nullptr;
  }
  return iso ? launch_fwd_seq<IsoB>(p, st) : launch_fwd_seq<DiagB>(p, st);
}

int kdn_scan_bwd(const KdnScanArgs* a, kdn_stream_t stream) {
  Sizes s;
  if (!sizes_of(a, &s))
    return set_error(KDN_ERR_INVALID,
                     "kdn_scan_bwd: unsupported variant/precision or shape (K and V must be 128; a packed batch "
                     "needs B = 1, the bf16 precision and its kdn_varlen_plan table)");
  const bool iso = a->variant == KDN_ISO;
  const int mode = a->mode;
  if (mode != KDN_SCAN_FULL && mode != KDN_SCAN_BWD_STATE)
    return set_error(KDN_ERR_INVALID, "kdn_scan_bwd: mode %d is not a backward mode", mode);
  if (mode != KDN_SCAN_FULL && a->precision != KDN_PREC_BF16)
    return set_error(KDN_ERR_INVALID, "kdn_scan_bwd: the partial-pass modes need the bf16 precision");
  if (a->num_seqs > 0 && mode != KDN_SCAN_FULL)
    return set_error(KDN_ERR_INVALID, "kdn_scan_bwd: a packed batch runs mode 0 only");
  if (mode == KDN_SCAN_BWD_STATE) {
    if (!a->q || !a->k || !a->v || !a->g || !a->saved || !a->dO || !a->d_initial_state ||
        (iso ? !a->beta : !a->kappa))
      return set_error(KDN_ERR_INVALID, "kdn_scan_bwd: null input/output pointer");
  } else if (!a->q || !a->k || !a->v || !a->g || !a->saved || !a->dO || !a->dq || !a->dk || !a->dv || !a->dg ||
             (iso ? (!a->beta || !a->dbeta) : (!a->kappa || !a->dkappa))) {
    return set_error(KDN_ERR_INVALID, "kdn_scan_bwd: null input/output pointer");
  }
  if (!a->workspace || a->workspace_bytes < kHeader + s.dh + s.dbg_bwd)
    return set_error(KDN_ERR_WORKSPACE, "kdn_scan_bwd: workspace too small");
  ScanParams p;
  int rc = fill_params(a, s, &p);
  if (rc != KDN_OK) return rc;
  char* ws = static_cast<char*>(a->workspace);
  p.status = reinterpret_cast<int*>(ws);
  p.dh = ws + kHeader;
  p.dbg = ws + kHeader + s.dh;
  p.dbg_stride = s.bwd_stride;
  const cudaStream_t st = (cudaStream_t)stream;
  if (reset_status(p.status, st, "kdn_scan_bwd: status reset") != KDN_OK) return KDN_ERR_CUDA;
  if (a->precision == KDN_PREC_FP32) return iso ? launch_bwd<IsoF>(p, st) : launch_bwd<DiagF>(p, st);
  if (!iso) p.g = reinterpret_cast<const float*>(static_cast<const char*>(a->saved) + kHeader + s.rec + s.h);
  if (mode == KDN_SCAN_BWD_STATE) return iso ? launch_bwd_state<IsoB>(p, st) : launch_bwd_state<DiagB>(p, st);
  if (iso) return launch_bwd<IsoB>(p, st);
  rc = launch_bwd<DiagB>(p, st);
  if (rc != KDN_OK) return rc;
  // cotangent of the 64-local prefix -> the boundary's 32-local one
  const int64_t HK4 = a->H * a->K / 4, NB64 = (a->T + 63) / 64, n = a->B * NB64 * HK4;
  if (p.vl.on()) {
    const int64_t nv = s.NT * HK4;
    gate_fold_varlen_kernel<<<grid_for(nv), 256, 0, st>>>(reinterpret_cast<float4*>(a->dg), p.vl, HK4, nv);
  } else {
    gate_fold_kernel<<<grid_for(n), 256, 0, st>>>(reinterpret_cast<float4*>(a->dg), a->T, HK4, NB64, n);
  }
  return check_launch("gate_fold_kernel");
}

}  // extern "C"
