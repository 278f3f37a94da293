"""B200-native (sm_100a) Veda block-sparse attention.

A drop-in for the Veda sparse-attention hot path of veda-sparse/Miowtion:
`attention.SparseStudent` is the pluggable `AttentionFn`; `kernels` mirrors
the reference's FA4 backend (`miowtion/kernels/fa4.py`); `tiling`, `mask`,
`predictor` and `plan` mirror `miowtion/veda/*`. The compute runs in the
C-ABI library `libveda_b200.so` (include/veda_b200.h).
"""

__all__ = ['attention', 'kernels', 'mask', 'plan', 'predictor', 'tiling']
