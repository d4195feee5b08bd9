"""Diagonal q / k normalisation (``_diag_kdn_normalize``,
diag_kdn_chunk.py:2162): bit-exact parity.

* CPU: the oracle's float32 restatement (``oracle.diag_normalize`` and
  ``diag_normalize_backward``) reproduces, bit for bit, the reference's own
  kernels run on a B200 (``tests/golden/diag_norm.npz``, made by
  ``tests/golden/make_norm_golden.py``).
* GPU: ``kdn_b200.diag_kdn_chunk._diag_kdn_normalize`` (the CUDA kernels
  through the C ABI) reproduces the fixture bit for bit, and the oracle on
  larger seeded cases; its validation raises the reference's exceptions.
The bar is bit equality of every output, bf16 and fp32 alike.
"""
import os

import numpy as np
import pytest
import torch

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "diag_norm.npz")


def cases():
    if not os.path.exists(GOLDEN):
        return []
    z = np.load(GOLDEN)
    return sorted({k[: -len("_meta")] for k in z.files if k.endswith("_meta")})


def load_case(name):
    z = np.load(GOLDEN)
    B, T, H, K, is_bf16, pq, pg, pm = (int(v) for v in z[name + "_meta"])
    dtype = torch.bfloat16 if is_bf16 else torch.float32

    def get(key, dt):
        a = z.get(name + "_" + key)
        if a is None:
            return None
        t = torch.from_numpy(a.copy())
        return t.view(torch.bfloat16) if dt == torch.bfloat16 else t

    d = {"q": get("q", dtype), "k": get("k", dtype), "q_memory": get("q_memory", torch.bfloat16),
         "k_gain": get("k_gain", torch.float32), "k_memory": get("k_memory", torch.bfloat16),
         "dq": get("dq", dtype), "dk": get("dk", dtype), "d_q_memory": get("d_q_memory", torch.bfloat16),
         "d_k_gain": get("d_k_gain", torch.float32), "d_k_memory": get("d_k_memory", torch.bfloat16)}
    return d


def bits_equal(x, ref):
    x, ref = x.detach().cpu(), ref.detach().cpu()
    if x.dtype != ref.dtype or x.shape != ref.shape:
        return False
    iv = torch.int16 if x.dtype == torch.bfloat16 else torch.int32
    return torch.equal(x.contiguous().view(iv), ref.contiguous().view(iv))


def test_golden_fixture_present():
    assert cases(), "tests/golden/diag_norm.npz is missing (tests/golden/make_norm_golden.py makes it on a GPU)"


@pytest.mark.parametrize("name", cases())
def test_oracle_matches_reference_bit_for_bit(name):
    d = load_case(name)
    q_memory, k_gain, k_memory, q_norm, k_norm = oracle.diag_normalize(d["q"], d["k"])
    assert bits_equal(q_memory, d["q_memory"])
    assert bits_equal(k_gain, d["k_gain"])
    assert bits_equal(k_memory, d["k_memory"])
    dq, dk = oracle.diag_normalize_backward(d["q"], d["k"], d["d_q_memory"], d["d_k_gain"], d["d_k_memory"],
                                            q_norm, k_norm)
    for got, ref in ((dq, d["dq"]), (dk, d["dk"])):
        assert (got is None) == (ref is None)
        if ref is not None:
            assert bits_equal(got, ref)


def run_ours(q, k, cots):
    from kdn_b200.diag_kdn_chunk import _diag_kdn_normalize

    ql, kl = q.cuda().requires_grad_(True), k.cuda().requires_grad_(True)
    outs = _diag_kdn_normalize(ql, kl)
    used = [(o, c.cuda()) for o, c in zip(outs, cots) if c is not None]
    torch.autograd.backward([o for o, _ in used], [c for _, c in used])
    return outs, ql.grad, kl.grad


@pytest.mark.gpu
@pytest.mark.parametrize("name", cases())
def test_kernels_match_reference_bit_for_bit(name):
    d = load_case(name)
    (q_memory, k_gain, k_memory), dq, dk = run_ours(d["q"], d["k"], (d["d_q_memory"], d["d_k_gain"], d["d_k_memory"]))
    assert bits_equal(q_memory, d["q_memory"])
    assert bits_equal(k_gain, d["k_gain"])
    assert bits_equal(k_memory, d["k_memory"])
    for got, ref in ((dq, d["dq"]), (dk, d["dk"])):
        assert (got is None) == (ref is None)
        if ref is not None:
            assert bits_equal(got, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,K,dtype", [(4, 256, 18, 128, torch.bfloat16), (1, 300, 5, 64, torch.bfloat16),
                                           (2, 100, 3, 128, torch.float32), (1, 7, 1, 128, torch.bfloat16),
                                           (1, 3, 4, 64, torch.float32)])
def test_kernels_match_oracle_bit_for_bit(B, T, H, K, dtype):
    gen = torch.Generator().manual_seed(B * 1000 + T + K)
    scale = torch.exp2(torch.randint(-6, 7, (B, T, H, 1), generator=gen).float())
    q = (torch.randn(B, T, H, K, generator=gen) * scale).to(dtype)
    k = (torch.randn(B, T, H, K, generator=gen) / scale).to(dtype)
    cots = (torch.randn(B, T, H, K, generator=gen).bfloat16(), torch.randn(B, T, H, K, generator=gen),
            torch.randn(B, T, H, K, generator=gen).bfloat16())
    (q_memory, k_gain, k_memory), dq, dk = run_ours(q, k, cots)
    ref = oracle.diag_normalize(q, k)
    assert bits_equal(q_memory, ref[0]) and bits_equal(k_gain, ref[1]) and bits_equal(k_memory, ref[2])
    rdq, rdk = oracle.diag_normalize_backward(q, k, *cots, ref[3], ref[4])
    assert bits_equal(dq, rdq) and bits_equal(dk, rdk)


@pytest.mark.gpu
def test_validation_matches_reference_messages():
    from kdn_b200.diag_kdn_chunk import _diag_kdn_normalize

    q = torch.randn(1, 4, 2, 128, device="cuda").bfloat16()
    with pytest.raises(ValueError, match="rank 4"):
        _diag_kdn_normalize(q[0], q[0])
    with pytest.raises(TypeError, match="BF16 or FP32"):
        _diag_kdn_normalize(q.half(), q.half())
    with pytest.raises(ValueError, match="matching dtype and grad mode"):
        _diag_kdn_normalize(q, q.float())
    with pytest.raises(ValueError, match="K in"):
        _diag_kdn_normalize(q[..., :96].contiguous(), q[..., :96].contiguous())
    with pytest.raises(ValueError, match="contiguous"):
        _diag_kdn_normalize(q.transpose(1, 2), q.transpose(1, 2))
