"""B200-native (sm_100a) Int8-weight LoRA linear for Reels.jl's low-VRAM path.

The compute lives in libreels_lowvram.so (include/reels_lowvram.h); this
package is the Python-side mirror of the reference's layer API
(:mod:`reels_b200.lowvram`) and its data-parallel gradient all-reduce
(:mod:`reels_b200.distributed`).
"""
from .lowvram import (  # noqa: F401
    DenseLayer,
    FrozenLinearFunction,
    LayerNormModulateFunction,
    GeluFeedForwardFunction,
    LoRALinear,
    LoRALinearFunction,
    QuantizedMatrix,
    check_device_status,
    dropout_mask,
    frozen_weight_transfer,
    gated_residual,
    gated_residual_backward,
    layernorm_modulate,
    layernorm_modulate_backward,
    linear,
    lora_backward,
    lora_forward,
    lora_forward_gelu,
    lora_parameters,
    materialize_weight,
    merged_weight,
    quantize_frozen_matrix,
    saved_buffer,
    set_adapter_enabled,
    weight_mul,
    weight_transpose_mul,
)

__version__ = "0.1.0"
