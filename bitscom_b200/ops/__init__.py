"""Low-level ops: Philox RNG restatement and sync-free quantise/pack helpers."""

from .philox import philox4x32_10, uniforms_for_elements
from .quant import pack_codes, quantize_codes, quantize_pack, unpack_dequant

__all__ = ["philox4x32_10", "uniforms_for_elements", "pack_codes", "quantize_codes", "quantize_pack", "unpack_dequant"]
