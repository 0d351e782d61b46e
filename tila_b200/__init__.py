"""B200 (sm_100a) execution backend for Tila's typed TIR.

Importing this package installs the backend into the installed Tila runtime:
launches of ``@ti.jit`` kernels on CUDA tensors are code-generated to CUDA
C++, compiled with NVRTC for sm_100a and launched through the native C ABI
(``libtila_b200.so``).  CPU arrays still run on Tila's NumPy interpreter.
"""

from ._reference import tila
from .plugin import B200, install, installed, uninstall
from .backend import check_device_errors, program_range, read_device_errors, generated_source

install()

__all__ = ["tila", "B200", "install", "uninstall", "installed", "program_range",
           "read_device_errors", "check_device_errors", "generated_source"]
