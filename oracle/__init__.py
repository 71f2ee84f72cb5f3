"""Parity checker for the SAM 3 PE backbone path (test infrastructure only).

Two CPU libraries, loaded through ctypes by `oracle.binding`:

* ``liboracle.so``      -- C restatement of the reference kernels (oracle.c);
* ``_ref/libsam3ref.so`` -- the reference's own sam3_kernels.cl compiled as
  host C++ through ocl_shim.hpp (built only where the reference tree exists).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs use
this package. The product (i.sam3.opencl_b200/) never imports it.
"""
