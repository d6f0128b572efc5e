"""Prints the compiler and linker flags of a torch C++ extension for this
interpreter's torch (used by the Makefile to build _hcops_torch.so)."""

import sys
import sysconfig

import torch
from torch.utils import cpp_extension

what = sys.argv[1] if len(sys.argv) > 1 else "cflags"
if what == "cflags":
    incs = cpp_extension.include_paths() + [sysconfig.get_paths()["include"], "/usr/local/cuda/include"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    print(" ".join(f"-I{p}" for p in incs), f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H")
else:
    libs = cpp_extension.library_paths()
    print(" ".join(f"-L{p}" for p in libs), "-lc10 -lc10_cuda -ltorch -ltorch_cpu -ltorch_cuda -ltorch_python")
