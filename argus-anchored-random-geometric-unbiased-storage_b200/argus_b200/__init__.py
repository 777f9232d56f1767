"""argus_b200: B200-native (sm_100a) implementation of ARGUS's tiered-KV hot path.

Drop-in for the reference package's surface (argus_cache 0.1.8, argus_cache/__init__.py:1-43): the
same module layout (core.quantization, core.triton_kernels, core.memory_manager,
models.attention_wrapper) and the same exported names, on CUDA tensors, backed by libargus_b200.so
(hand-written sm_100a kernels behind a C ABI, include/argus_b200.h).
"""
__version__ = "0.1.0"


def __getattr__(name):
    # lazy: importing the package must not require a GPU
    if name == "PagedDynamicQuantizedCache":
        from .models.attention_wrapper import PagedDynamicQuantizedCache
        return PagedDynamicQuantizedCache
    if name == "PagedDynamicKVCache":
        from .core.memory_manager import PagedDynamicKVCache
        return PagedDynamicKVCache
    if name == "patch_model_with_argus":
        return patch_model_with_argus
    raise AttributeError(name)


def patch_model_with_argus(model, page_size=4096, max_active_pages=2, max_fp8_pages=2, max_int8_pages=2,
                           max_int4_pages=2, max_int2_pages=2, max_one_bit_pages=2, sink_tokens=4):
    """Makes model.generate() use a PagedDynamicQuantizedCache (argus_cache/__init__.py:4-36)."""
    from .models.attention_wrapper import PagedDynamicQuantizedCache

    original_prep = model.prepare_inputs_for_generation

    def prepare_inputs_for_generation_argus(*args, **kwargs):
        if kwargs.get("past_key_values", None) is None:
            kwargs["past_key_values"] = PagedDynamicQuantizedCache(
                page_size=page_size, max_active_pages=max_active_pages, max_fp8_pages=max_fp8_pages,
                max_int8_pages=max_int8_pages, max_int4_pages=max_int4_pages, max_int2_pages=max_int2_pages,
                max_one_bit_pages=max_one_bit_pages, sink_tokens=sink_tokens)
        return original_prep(*args, **kwargs)

    model.prepare_inputs_for_generation = prepare_inputs_for_generation_argus
    return model


__all__ = ["PagedDynamicQuantizedCache", "PagedDynamicKVCache", "patch_model_with_argus"]
