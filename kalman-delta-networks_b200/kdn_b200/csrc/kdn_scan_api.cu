// C ABI of the chunked memory scan: argument validation, caller-owned saved
// state and workspace layout, and dispatch to the kernel instantiations.
#include <math.h>

#include "kdn_scan.cuh"

namespace kdn {

template <class CF> int launch_fwd(const ScanParams&, cudaStream_t);
template <class CF> int launch_bwd(const ScanParams&, cudaStream_t);
template <class CF> size_t fwd_dbg_bytes();
template <class CF> size_t state_bytes();
template <class CF> size_t chunk_bytes();

using IsoB = Cfg<true, 64, bf16>;
using IsoF = Cfg<true, 64, float>;
using DiagB = Cfg<false, 32, bf16>;
using DiagF = Cfg<false, 32, float>;

namespace {

struct Sizes {
  int64_t C, NT, BH, op;  // chunk, chunks, streams, bytes per state element
  size_t tq, h, dh, dbg_fwd, dbg_bwd;
};

bool sizes_of(const KdnScanArgs* a, Sizes* s) {
  if (!a || (a->variant != KDN_ISO && a->variant != KDN_DIAG) ||
      (a->precision != KDN_PREC_BF16 && a->precision != KDN_PREC_FP32))
    return false;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->K != kKD || a->V != kVD) return false;
  s->C = a->variant == KDN_ISO ? 64 : 32;
  s->NT = (a->T + s->C - 1) / s->C;
  s->BH = a->B * a->H;
  s->op = a->precision == KDN_PREC_FP32 ? 4 : 2;
  s->tq = align_up((size_t)s->op * s->BH * s->NT * s->C * s->C, 256);
  s->h = align_up((size_t)s->op * s->BH * s->NT * kKD * kVD, 256);
  s->dh = s->h;
  s->dbg_fwd = s->dbg_bwd = 0;
  if (a->precision == KDN_PREC_FP32) {
    const bool iso = a->variant == KDN_ISO;
    const size_t f = iso ? fwd_dbg_bytes<IsoF>() : fwd_dbg_bytes<DiagF>();
    const size_t st = iso ? state_bytes<IsoF>() : state_bytes<DiagF>();
    const size_t ck = iso ? chunk_bytes<IsoF>() : chunk_bytes<DiagF>();
    s->dbg_fwd = align_up(f * 2 * s->BH, 256);
    // both backward kernels index per-CTA slices with one stride
    s->dbg_bwd = align_up((st > ck ? st : ck) * (size_t)(s->NT > 2 ? s->NT : 2) * s->BH, 256);
  }
  return true;
}

int fill_params(const KdnScanArgs* a, const Sizes& s, ScanParams* p) {
  if (!(isfinite(a->scale))) return set_error(KDN_ERR_INVALID, "kdn_scan: scale must be finite");
  if (a->T > (1ll << 30) || s.BH > 65535) return set_error(KDN_ERR_INVALID, "kdn_scan: size too large");
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
  p->Tsave = sv;
  p->Qsave = sv + s.tq;
  p->h = sv + 2 * s.tq;
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
  p->scale = a->scale;
  return KDN_OK;
}

}  // namespace
}  // namespace kdn

using namespace kdn;

extern "C" {

size_t kdn_scan_saved_bytes(const KdnScanArgs* a) {
  Sizes s;
  if (!sizes_of(a, &s)) return 0;
  return 2 * s.tq + s.h;
}

size_t kdn_scan_workspace_bytes(const KdnScanArgs* a) {
  Sizes s;
  if (!sizes_of(a, &s)) return 0;
  const size_t bwd = s.dh + s.dbg_bwd;
  return bwd > s.dbg_fwd ? bwd : s.dbg_fwd;
}

int kdn_scan_fwd(const KdnScanArgs* a, kdn_stream_t stream) {
  Sizes s;
  if (!sizes_of(a, &s))
    return set_error(KDN_ERR_INVALID, "kdn_scan_fwd: unsupported variant/precision or shape (K and V must be 128)");
  if (!a->q || !a->k || !a->v || !a->g || !a->o || !a->saved ||
      (a->variant == KDN_ISO ? !a->beta : !a->kappa))
    return set_error(KDN_ERR_INVALID, "kdn_scan_fwd: null input/output pointer");
  if (s.dbg_fwd && (!a->workspace || a->workspace_bytes < s.dbg_fwd))
    return set_error(KDN_ERR_WORKSPACE, "kdn_scan_fwd: workspace too small");
  ScanParams p;
  int rc = fill_params(a, s, &p);
  if (rc != KDN_OK) return rc;
  p.dbg = static_cast<char*>(a->workspace);
  const bool iso = a->variant == KDN_ISO;
  if (a->precision == KDN_PREC_FP32) {
    p.dbg_stride = iso ? fwd_dbg_bytes<IsoF>() : fwd_dbg_bytes<DiagF>();
    return iso ? launch_fwd<IsoF>(p, (cudaStream_t)stream) : launch_fwd<DiagF>(p, (cudaStream_t)stream);
  }
  return iso ? launch_fwd<IsoB>(p, (cudaStream_t)stream) : launch_fwd<DiagB>(p, (cudaStream_t)stream);
}

int kdn_scan_bwd(const KdnScanArgs* a, kdn_stream_t stream) {
  Sizes s;
  if (!sizes_of(a, &s))
    return set_error(KDN_ERR_INVALID, "kdn_scan_bwd: unsupported variant/precision or shape (K and V must be 128)");
  const bool iso = a->variant == KDN_ISO;
  if (!a->q || !a->k || !a->v || !a->g || !a->saved || !a->dO || !a->dq || !a->dk || !a->dv || !a->dg ||
      (iso ? (!a->beta || !a->dbeta) : (!a->kappa || !a->dkappa)))
    return set_error(KDN_ERR_INVALID, "kdn_scan_bwd: null input/output pointer");
  if (!a->workspace || a->workspace_bytes < s.dh + s.dbg_bwd)
    return set_error(KDN_ERR_WORKSPACE, "kdn_scan_bwd: workspace too small");
  ScanParams p;
  int rc = fill_params(a, s, &p);
  if (rc != KDN_OK) return rc;
  p.dh = a->workspace;
  p.dbg = static_cast<char*>(a->workspace) + s.dh;
  if (a->precision == KDN_PREC_FP32) {
    // both backward kernels use the same per-CTA stride bound
    const size_t st = iso ? state_bytes<IsoF>() : state_bytes<DiagF>();
    const size_t ck = iso ? chunk_bytes<IsoF>() : chunk_bytes<DiagF>();
    p.dbg_stride = st > ck ? st : ck;
    return iso ? launch_bwd<IsoF>(p, (cudaStream_t)stream) : launch_bwd<DiagF>(p, (cudaStream_t)stream);
  }
  return iso ? launch_bwd<IsoB>(p, (cudaStream_t)stream) : launch_bwd<DiagB>(p, (cudaStream_t)stream);
}

}  // extern "C"
