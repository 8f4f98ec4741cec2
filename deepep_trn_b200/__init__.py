"""deepep_trn_b200: a deep_ep-compatible MoE expert-parallel communication library for B200.

Hand-written sm_100a kernels move tokens between the GPUs of one NVLink 5 /
NVSwitch node through peer-mapped memory; PyTorch is the framework layer.
"""
from .buffer import Buffer
from .handles import Config, DispatchHandle, EventOverlap, LowLatencyHandle
from .utils.codec import RowCodec
from .utils.layout import get_dispatch_layout

__all__ = ['Buffer', 'Config', 'DispatchHandle', 'EventOverlap', 'LowLatencyHandle', 'RowCodec',
           'get_dispatch_layout']
__version__ = '0.1.0'
