"""nelisp_cuda -- Python host side of libnelisp_cuda.

* ``_lib``     : ctypes binding of the C ABI (include/nelisp_cuda.h)
* ``host``     : in-process API with the call shapes of lisp/nelisp-gpu-server.el
* ``server``   : subprocess client of the protocol server (bin/nelisp-cuserver)
* ``protocol`` : the server wire encoders
* ``f32codec`` : the reference's float32 wire codec
* ``dev``      : typed entry points on device tensors
* ``build``    : compiles the library, the server and the CLIs in-tree
"""
from ._lib import LIB_PATH, BIN_DIR, NlError, load  # noqa: F401
