"""ctypes binding of ``libglmkv.so`` (the C ABI in ``include/glmkv.h``).

The library is built in-tree by ``kern-glm53_b200/glmkv/build.py``; loading fails loudly when it is
missing (there is no other implementation to fall back to).
"""
import ctypes
import pathlib

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libglmkv.so"
CUBIN_PATH = pathlib.Path(__file__).resolve().parent / "glm_glue_b200.cubin"

# Exported symbols and their ctypes signatures: (name, argtypes). Every launcher returns int.
P, I = ctypes.c_void_p, ctypes.c_int
SIGNATURES = {
    "glmkv_plan": [P, P, I, P, P, P, P, P, P, I, P],
    "glmkv_mla_prep": [P, I, P, P, P, P, P, P, P, P, P, P, P, I, I, P],
    "glmkv_mla_prep_fp8": [P, I, P, P, P, P, P, P, P, P, P, P, P, I, I, P],
    "glmkv_idx_gather": [P, P, I, P, I, P, P, P],
    "glmkv_kv_dequant": [P, P, I, P, I, P, P],
    "glmkv_mark_rows": [P, P, P, I, P, I, P],
    "glmkv_topk_stream_mark": [P, P, P, P, I, P, P, I, P],
    "glmkv_kv_dequant_marked": [P, P, I, P, I, P, P, P],
    "glmkv_topk_stream": [P, P, P, P, I, P],
    "glmkv_topk_slots": [P, P, I, P, P, P, I, P],
    "glmkv_q_post": [P, I, P, P, P, P, P, P, I, I, P],
    "glmkv_add_rms_quant": [P, P, P, P, P, P, I, I, P],
    "glmkv_quant": [P, I, P, P, I, I, I, P],
    "glmkv_mqa_logits_paged": [P, P, I, P, I, P, P, P, P, I, I, P],
    "glmkv_launch_shape": [ctypes.c_char_p, I, P, P, P],
    "glmkv_selftest_wait": [ctypes.c_uint64, P, P],
    "glmkv_fault_flags": [P, I],
    "glmkv_strerror": [I],
    "glmkv_abi_version": [],
}

OK, ERR_ARG, ERR_ALIGN, ERR_DEVICE, ERR_LAUNCH = range(5)

_lib = None


class GlmKvError(RuntimeError):
    """A launcher returned a non-zero status."""

    def __init__(self, op, code):
        self.op, self.code = op, code
        super().__init__(f"{op}: {strerror(code)} (code {code})")


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `python kern-glm53_b200/glmkv/build.py` "
                              "(the CUDA kernels are the only implementation)")
        l = ctypes.CDLL(str(LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(l, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_char_p if name == "glmkv_strerror" else ctypes.c_int
        _lib = l
    return _lib


def strerror(code):
    return lib().glmkv_strerror(int(code)).decode()


def call(name, *args):
    rc = getattr(lib(), name)(*args)
    if rc != OK:
        raise GlmKvError(name, rc)


def launch_shape(entry, T=0):
    """(grid, block, dynamic smem bytes) libglmkv launches `entry` with on the current device."""
    g, b, s = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    call("glmkv_launch_shape", entry.encode(), int(T), ctypes.byref(g), ctypes.byref(b), ctypes.byref(s))
    return g.value, b.value, s.value


def fault_flags(clear=True):
    """The module's device fault bits on the current device (1: a wait timed out, 2: a bad page, 4: a pick
    past the mark bitmap)."""
    v = ctypes.c_uint32(0)
    call("glmkv_fault_flags", ctypes.byref(v), int(bool(clear)))
    return v.value
