"""dwarf_v2_b200 -- B200 (sm_100a) inference engine for the DWARF-v2 sparse-attention prefill path.

Drop-in modules mirroring the reference's public API:

* ``dwarf_v2_b200.causal_ema_scan``            (kernels/causal_ema_scan.py)
* ``dwarf_v2_b200.dsqg_attention_v22``         (kernels/dsqg_attention_v22.py)
* ``dwarf_v2_b200.hierarchical_sparse_attn_v18_hisa``
                                               (kernels/hierarchical_sparse_attn_v18_hisa.py)
* ``dwarf_v2_b200.model``                      (model construction of train/train_dwarf.py)

All device work runs in hand-written CUDA kernels behind the C ABI declared in
include/dwarf_b200.h (``libdwarf_b200.so``), plus cuBLAS GEMMs through torch.
"""

__version__ = "0.1.0"
