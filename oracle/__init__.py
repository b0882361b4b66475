"""CPU oracle for the DWARF-v2 prefill path -- TEST INFRASTRUCTURE ONLY.

These modules restate the reference algorithms (Lanerra/dwarf-v2, the files
kernels/causal_ema_scan.py, kernels/dsqg_attention_v22.py,
kernels/hierarchical_sparse_attn_v18_hisa.py and train/train_dwarf.py) in plain
numpy / CPU torch so that the CUDA engine can be checked against them. Each
function cites the reference lines it follows.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this package, and only as the checker or the timed CPU
baseline. The engine in dwarf_v2_b200/ never imports it.
"""
