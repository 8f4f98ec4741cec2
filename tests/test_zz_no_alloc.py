"""The allocation-free layout entry point, called through its exported C symbol.

This is for callers of the library that must not allocate device memory while
they run (engines with pre-planned memory, plugin enqueue paths, code outside
PyTorch without a caching allocator): the entry point keeps its scratch in an
array compiled into the library. The tests check its outputs against the
regular layout op on calls in a row, so later calls also show that the shared
scratch was left clean by earlier ones; the first call of a fresh process runs
on a non-blocking stream, which is not ordered with the legacy default stream.
The file is collected last.
"""
import ctypes
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason='needs CUDA')

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _symbol():
    from deepep_trn_b200.ops import load
    mod = load()  # the regular extension; the C symbol lives in the same shared object
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.b200ep_dispatch_layout_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _compare_calls(cases, stream):
    """Run the regular op and the entry point on every case (on ``stream``) and compare."""
    from deepep_trn_b200.ops import load
    from deepep_trn_b200.utils.testing import make_routing
    C = load()
    fn = _symbol()
    dev = torch.device('cuda', 0)
    with torch.cuda.stream(stream):
        for call, (kind, T, E, K, R) in enumerate(cases):
            if T == 0:
                idx = torch.empty(0, K, dtype=torch.int64)
            else:
                idx, _ = make_routing(kind, T, E, K, R, 0, seed=call)
            d_idx = idx.to(dev, non_blocking=False)
            T = idx.shape[0]
            out = (torch.full((R,), -7, dtype=torch.int32, device=dev),
                   torch.full((E,), -7, dtype=torch.int32, device=dev),
                   torch.ones(T, R, dtype=torch.bool, device=dev))
            # the entry point first: in a fresh process this is the call that sets up the scratch
            rc = fn(d_idx.data_ptr(), T, K, E, R, out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(),
                    stream.cuda_stream)
            assert rc == 0, rc
            ref = (torch.empty(R, dtype=torch.int32, device=dev), torch.empty(E, dtype=torch.int32, device=dev),
                   torch.empty(T, R, dtype=torch.bool, device=dev))
            C.layout(d_idx, E, R, *ref, torch.zeros(R + E + 1, dtype=torch.int32, device=dev))
            stream.synchronize()
            for a, b in zip(out, ref):
                assert torch.equal(a, b), (kind, T, a, b)
            if T == 0:
                assert int(out[0].abs().sum()) == 0 and int(out[1].abs().sum()) == 0


CASES = [('random', 4096, 256, 8, 8), ('masked', 777, 64, 6, 4), ('random', 0, 256, 8, 8),
         ('hot_rank0', 1000, 256, 8, 8)]


@needs_cuda
def test_noalloc_layout_matches_regular_entry_point():
    _compare_calls(CASES, torch.cuda.current_stream())


@needs_cuda
def test_noalloc_first_call_on_nonblocking_stream_in_fresh_process():
    code = ('import sys, torch; sys.path.insert(0, %r); sys.path.insert(0, %r); '
            'import test_zz_no_alloc as t; t._compare_calls(t.CASES, torch.cuda.Stream()); print("fresh OK")'
            % (ROOT, os.path.join(ROOT, 'tests')))
    p = subprocess.run([sys.executable, '-c', code], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert p.returncode == 0 and 'fresh OK' in p.stdout, p.stdout + p.stderr


@needs_cuda
def test_noalloc_layout_rejects_sizes_beyond_limit():
    fn = _symbol()
    rc = fn(None, 16, 8, 8192, 8, None, None, None, None)
    assert rc == -2
