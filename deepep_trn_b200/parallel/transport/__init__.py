from .base import Transport
from .gloo import GlooTransport
from .nccl import NcclTransport

__all__ = ['Transport', 'GlooTransport', 'NcclTransport']
