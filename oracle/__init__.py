"""Test oracles for the KV-cache path (test infrastructure only; never imported by the product).

``oracle.cpu``  -- ctypes wrapper over the C restatement ``glm_oracle.c``.
``oracle.ref``  -- ctypes wrapper over the reference's own glue kernels built from source
                   (``oracle/_ref/libglmref.so``), used on the GPU as the bit-exact oracle.
"""
