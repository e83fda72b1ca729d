"""lagunalab_b200: the Laguna MoE block and the fused 8-bit KV decode attention on B200.

The public surface mirrors lagunaLab's ``laguna_mlx`` package (``laguna``, ``cache``,
``q8_attn``, ``streaming``, ``hooks``); the arithmetic runs in the sm_100a kernels of
``liblaguna_b200.so`` (C ABI in ``include/laguna_b200.h``), called through ``ops``.
"""
__version__ = "0.1.0"
