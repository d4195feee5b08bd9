"""kdn_b200 -- B200 (sm_100a) kernels for the Kalman Delta Network scan.

Drop-in operators with the reference ``lit_gpt.kdn_ops`` signatures:

* ``kdn_b200.iso_kdn_chunk``: ``iso_kdn_gain``, ``_chunk_kda_precumsum_paired``
* ``kdn_b200.diag_kdn_chunk``: ``_diag_kdn_gain``, ``chunk_kalman``,
  ``_diag_kdn_frontend_precumsum_paired``

The compute runs in ``lib/libkdn_b200.so`` (C ABI, ``include/kdn_b200.h``).
"""
from . import _native  # noqa: F401

__version__ = "0.1.0"
