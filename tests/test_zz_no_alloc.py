"""The allocation-free layout entry point, called through its exported C symbol.

This is for callers of the library that must not allocate device memory while
they run (engines with pre-planned memory, plugin enqueue paths, code outside
PyTorch without a caching allocator): the entry point keeps its scratch in an
array compiled into the library. The test checks its outputs against the
regular layout op on two calls in a row, so the second call also shows that the
shared scratch was left clean by the first. It lives in a file of its own that
pytest collects last.
"""
import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason='needs CUDA')

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _symbol():
    from deepep_trn_b200.ops import load
    load()  # the regular extension; the C symbol lives in the same shared object
    path = glob.glob(os.path.join(ROOT, 'deepep_trn_b200', '_C*.so'))[0]
    lib = ctypes.CDLL(path)
    fn = lib.b200ep_dispatch_layout_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return fn


@needs_cuda
def test_noalloc_layout_matches_regular_entry_point():
    from deepep_trn_b200.ops import load
    from deepep_trn_b200.utils.testing import make_routing
    C = load()
    fn = _symbol()
    dev = torch.device('cuda', 0)
    stream = torch.cuda.current_stream()
    for call, (kind, T, E, K, R) in enumerate([('random', 4096, 256, 8, 8), ('masked', 777, 64, 6, 4)]):
        idx, _ = make_routing(kind, T, E, K, R, 0, seed=call)
        d_idx = idx.to(dev)
        T = idx.shape[0]
        ref = (torch.empty(R, dtype=torch.int32, device=dev), torch.empty(E, dtype=torch.int32, device=dev),
               torch.empty(T, R, dtype=torch.bool, device=dev))
        C.layout(d_idx, E, R, *ref, torch.zeros(R + E + 1, dtype=torch.int32, device=dev))
        out = (torch.full((R,), -7, dtype=torch.int32, device=dev), torch.full((E,), -7, dtype=torch.int32, device=dev),
               torch.ones(T, R, dtype=torch.bool, device=dev))
        rc = fn(d_idx.data_ptr(), T, K, E, R, out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(),
                stream.cuda_stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        for a, b in zip(out, ref):
            assert torch.equal(a, b), (kind, a, b)


@needs_cuda
def test_noalloc_layout_rejects_sizes_beyond_limit():
    fn = _symbol()
    rc = fn(None, 16, 8, 8192, 8, None, None, None, None)
    assert rc == -2
