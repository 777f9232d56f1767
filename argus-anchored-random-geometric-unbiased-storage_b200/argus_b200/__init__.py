"""argus_b200: B200-native (sm_100a) implementation of ARGUS's tiered-KV hot path.

Drop-in for the reference package's surface (argus_cache 0.1.8): the same module layout
(core.quantization, core.triton_kernels, core.memory_manager, models.attention_wrapper) and
the same exported names, on CUDA tensors, backed by libargus_b200.so.
"""
__version__ = "0.1.0"
