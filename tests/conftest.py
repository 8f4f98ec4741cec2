import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200 / sm_100a)')


def free_port() -> int:
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def torchrun(script: str, nproc: int, *args, timeout: int = 600, env=None):
    """Run a tests/dist script under torchrun on 127.0.0.1; returns (returncode, output)."""
    cmd = [sys.executable, '-m', 'torch.distributed.run', '--nnodes', '1', '--nproc-per-node', str(nproc),
           '--master-addr', '127.0.0.1', '--master-port', str(free_port()),
           str(ROOT / 'tests' / 'dist' / script), *map(str, args)]
    e = dict(os.environ)
    e.setdefault('OMP_NUM_THREADS', '1')
    e['PYTHONPATH'] = str(ROOT) + os.pathsep + e.get('PYTHONPATH', '')
    if env:
        e.update(env)
    for _ in range(3):
        p = subprocess.run(['timeout', '-k', '30', str(timeout), *cmd], capture_output=True, text=True, env=e,
                           cwd=str(ROOT))
        out = p.stdout + p.stderr
        if p.returncode == 0 or 'EADDRINUSE' not in out:
            break
        # the rendezvous port was taken between probing and binding: retry on a fresh one
        cmd[cmd.index('--master-port') + 1] = str(free_port())
    return p.returncode, out


@pytest.fixture
def run_dist():
    return torchrun
