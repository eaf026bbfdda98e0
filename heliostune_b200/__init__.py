"""heliostune_b200: heliostune's FP16 matmul path, built for the NVIDIA B200 (sm_100a).

Configuration, enumeration and the bandit import neither torch nor the native library; the GPU
entry points (``kernel.matmul``, ``hopper_kernel.hopper_matmul``, ``action_expansion.launch``,
``fusion.rmsnorm``) load ``libheliostune_b200.so`` on first use and raise if it is missing.
"""

__version__ = "0.1.0"
