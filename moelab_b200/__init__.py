"""moelab_b200: B200-native (sm_100a) quantized MoE-layer forward for moe-lab.

The package is the `moe-lab_b200` component of this repository (Python module names cannot contain '-').
Variants live in moelab_b200/variants/cuda/*.py and follow moe-lab's variant contract
(META, W_BITS, prepare, run, dequant), so moelab/torch_backend.py:35-40 `load_variant(path)` loads them.
"""
__version__ = "0.1.0"
