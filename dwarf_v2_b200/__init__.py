"""dwarf_v2_b200 -- B200 (sm_100a) inference engine for the DWARF-v2 sparse-attention prefill path.

Drop-in modules mirroring the reference's public API:

* ``dwarf_v2_b200.causal_ema_scan``            (kernels/causal_ema_scan.py)
* ``dwarf_v2_b200.dsqg_attention_v22``         (kernels/dsqg_attention_v22.py)
* ``dwarf_v2_b200.hierarchical_sparse_attn_v18_hisa``
                                               (kernels/hierarchical_sparse_attn_v18_hisa.py)
* ``dwarf_v2_b200.model``                      (model construction of train/train_dwarf.py)

All device work runs in hand-written sm_100a CUDA kernels behind the C ABI
declared in include/dwarf_b200.h (``libdwarf_b200.so``): the attention, scan and
glue kernels and a tcgen05 GEMM with fused epilogues. A few projection GEMMs of
the DSQG and HISA modules still go through torch (cuBLAS).

``check_device_status(device=None)`` raises ``DeviceTimeoutError`` when a kernel
hit its bounded-wait limit since the last check (its outputs are then invalid).
"""

__version__ = "0.2.0"


def check_device_status(device=None) -> None:
    """Raise DeviceTimeoutError if a kernel recorded a timed-out wait (see ``_lib.check_device_status``)."""
    from . import _lib

    _lib.check_device_status(device)
