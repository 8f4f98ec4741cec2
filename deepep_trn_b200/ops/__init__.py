"""Thin Python wrappers over the sm_100a kernels (no torch fallbacks on CUDA tensors)."""
from ._ext import available, load
from .quant import quantize_fp8

__all__ = ['available', 'load', 'quantize_fp8']
