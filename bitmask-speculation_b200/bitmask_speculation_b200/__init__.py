"""B200-native (sm_100a) masked-selection path of bitmask-speculation.

Fused masked argmax + valid count, online-softmax inverse-CDF masked sampling
and batched K+1-row verification over packed grammar masks, as hand-written CUDA
behind a C ABI (``include/bms_b200.h``).  ``kernels.cuda`` mirrors the
reference's Python API; ``kernels._extension.load_extension`` is the drop-in for
the reference's native module.
"""

__version__ = "0.1.0"
