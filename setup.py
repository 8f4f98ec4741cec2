"""In-tree build of the sm_100a extension: ``python setup.py build_ext --inplace``.

The shared object lands next to the sources as ``deepep_trn_b200/_C*.so`` so it
travels with the repository snapshot; nothing is installed into site-packages.
"""
import os
from pathlib import Path

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / 'deepep_trn_b200' / 'csrc'
SOURCES = sorted(str(p.relative_to(ROOT)) for p in list(CSRC.glob('*.cu')) + list(CSRC.glob('*.cpp')))

NVCC_FLAGS = [
    '-gencode', 'arch=compute_100a,code=sm_100a',
    '-lineinfo', '-O3', '-std=c++17',
    '--expt-relaxed-constexpr', '--expt-extended-lambda',
    '-U__CUDA_NO_HALF_OPERATORS__', '-U__CUDA_NO_HALF_CONVERSIONS__',
    '-U__CUDA_NO_BFLOAT16_CONVERSIONS__', '-U__CUDA_NO_HALF2_OPERATORS__',
]
if os.environ.get('B200EP_PTXAS_VERBOSE'):
    NVCC_FLAGS.append('-Xptxas=-v')

setup(
    name='deepep_trn_b200',
    ext_modules=[CUDAExtension(
        name='deepep_trn_b200._C',
        sources=SOURCES,
        include_dirs=[str(CSRC)],
        extra_compile_args={'cxx': ['-O3', '-std=c++17'], 'nvcc': NVCC_FLAGS},
    )],
    cmdclass={'build_ext': BuildExtension.with_options(use_ninja=True)},
)
