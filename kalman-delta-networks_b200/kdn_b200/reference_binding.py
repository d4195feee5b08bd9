"""Load an installed copy of the reference (ngocbh/kalman-delta-networks) with
kdn_b200's operators bound in: the rebinding INTEGRATION.md section 1 shows,
done programmatically, so the reference's own model (``lit_gpt.model.GPT``,
its blocks, mixers, RMSNorm, SwiGLU MLP and fused cross-entropy) trains on
the B200 kernels.

Bound (when ``bind``): in ``lit_gpt.kdn_ops.iso_kdn_chunk`` ``iso_kdn_gain``,
``_chunk_kda_precumsum_paired``, ``_iso_kdn_gate_precumsum_paired`` and
``qkv_causal_conv1d``; in ``lit_gpt.kdn_ops.diag_kdn_chunk`` ``_diag_kdn_gain``,
``chunk_kalman``, ``_diag_kdn_frontend_precumsum_paired`` and
``_diag_kdn_normalize``; the mixers' ``FusedRMSNormGated`` and the diagonal
mixer's ``_fixed_short_conv``.

The reference's package ``__init__`` and ``lit_gpt.utils`` import its training
stack (lightning), which building and training the model does not need; the
package object is created without running ``__init__``, and ``lit_gpt.utils``
is a stand-in holding the one helper ``lit_gpt.config`` imports from it.
Modules load from ``<root>/lit_gpt`` in a fixed order (ops, bindings, mixers,
model) so that names imported at module import see the bound operators.
The bindings are process-wide (``sys.modules``).
"""
from __future__ import annotations

import importlib
import os
import sys
import types

_KDN_MODULES = ("lit_gpt.kdn_ops.iso_kdn_chunk", "lit_gpt.kdn_ops.diag_kdn_chunk", "lit_gpt.iso_kdn",
                "lit_gpt.diag_kdn", "lit_gpt.model", "lit_gpt.config")


def _find_multiple(n: int, k: int) -> int:
    """The smallest multiple of k that is >= n (what lit_gpt.config imports from lit_gpt.utils)."""
    return n if n % k == 0 else n + k - n % k


def load_reference(root: str, bind: bool = True) -> types.SimpleNamespace:
    """Import the reference's ``lit_gpt`` from ``root`` (the directory holding
    ``lit_gpt/``), with kdn_b200's operators bound in when ``bind``.  Returns
    a namespace with ``model`` (lit_gpt.model), ``config`` (lit_gpt.config),
    ``iso_kdn``, ``diag_kdn``, ``ops_iso``, ``ops_diag`` and
    ``FusedCrossEntropyLoss``."""
    path = os.path.join(os.path.abspath(root), "lit_gpt")
    if not os.path.isdir(path):
        raise FileNotFoundError(f"no lit_gpt package under {root}")
    pkg = sys.modules.get("lit_gpt")
    if pkg is None or list(getattr(pkg, "__path__", [])) != [path]:
        pkg = types.ModuleType("lit_gpt")
        pkg.__path__ = [path]
        sys.modules["lit_gpt"] = pkg
    if "lit_gpt.utils" not in sys.modules:
        utils = types.ModuleType("lit_gpt.utils")
        utils.find_multiple = _find_multiple
        sys.modules["lit_gpt.utils"] = utils
    for name in _KDN_MODULES:  # fresh imports, so the bindings below are the ones seen
        sys.modules.pop(name, None)

    ops_iso = importlib.import_module("lit_gpt.kdn_ops.iso_kdn_chunk")
    ops_diag = importlib.import_module("lit_gpt.kdn_ops.diag_kdn_chunk")
    if bind:
        from . import diag_kdn_chunk, iso_kdn_chunk, short_conv

        ops_iso.iso_kdn_gain = iso_kdn_chunk.iso_kdn_gain
        ops_iso._chunk_kda_precumsum_paired = iso_kdn_chunk._chunk_kda_precumsum_paired
        ops_iso._iso_kdn_gate_precumsum_paired = iso_kdn_chunk._iso_kdn_gate_precumsum_paired
        ops_iso.qkv_causal_conv1d = short_conv.qkv_causal_conv1d
        for name in ("_diag_kdn_gain", "chunk_kalman", "_diag_kdn_frontend_precumsum_paired", "_diag_kdn_normalize"):
            setattr(ops_diag, name, getattr(diag_kdn_chunk, name))
    iso_kdn = importlib.import_module("lit_gpt.iso_kdn")
    diag_kdn = importlib.import_module("lit_gpt.diag_kdn")
    if bind:
        from .norm_gated import FusedRMSNormGated
        from .short_conv import fixed_short_conv

        iso_kdn.FusedRMSNormGated = FusedRMSNormGated
        diag_kdn.FusedRMSNormGated = FusedRMSNormGated
        diag_kdn._fixed_short_conv = fixed_short_conv
    model = importlib.import_module("lit_gpt.model")  # imports lit_gpt.config, as the package __init__ does
    config = sys.modules["lit_gpt.config"]
    fce = importlib.import_module("lit_gpt.fused_cross_entropy")
    return types.SimpleNamespace(model=model, config=config, iso_kdn=iso_kdn, diag_kdn=diag_kdn, ops_iso=ops_iso,
                                 ops_diag=ops_diag, FusedCrossEntropyLoss=fce.FusedCrossEntropyLoss)


__all__ = ("load_reference",)
