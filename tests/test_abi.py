"""The C ABI without a GPU: the library loads, exports every symbol include/glmkv.h declares, and
rejects invalid arguments on the host (before any CUDA call)."""
import ctypes
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "glmkv.h"


def declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^(?:int|const char\*)\s+(glmkv_\w+)\s*\(", text, flags=re.M)


def _has_cuda_device():
    try:
        import torch
        return torch.cuda.is_available()
    except ImportError:
        return False


def test_header_declares_the_manifest_ops():
    names = set(declared())
    assert {"glmkv_plan", "glmkv_mla_prep", "glmkv_mla_prep_fp8", "glmkv_idx_gather", "glmkv_kv_dequant",
            "glmkv_topk_stream", "glmkv_topk_slots"} <= names


def test_library_exports_every_declared_symbol(built_lib):
    lib = ctypes.CDLL(str(built_lib))
    for name in declared():
        assert hasattr(lib, name), name
    import glmkv
    assert set(declared()) == set(glmkv._lib.SIGNATURES)
    assert glmkv.lib().glmkv_abi_version() == 102


def test_host_side_argument_checks(built_lib):
    import glmkv
    from glmkv import _lib

    L = glmkv.lib()
    A = 0x10000  # an aligned, never dereferenced address: every call below returns before any CUDA call
    assert L.glmkv_plan(A, A, 0, A, A, A, A, A, A, 16, None) == _lib.ERR_ARG          # nseq < 1
    assert L.glmkv_plan(A, A, 1, A, A, A, A, A, A, -1, None) == _lib.ERR_ARG          # T < 0
    assert L.glmkv_plan(A, A, 1, None, A, A, A, A, A, 16, None) == _lib.ERR_ARG       # null output
    assert L.glmkv_plan(A, A, 1, A, A, A, A, A, A, 0, None) == _lib.OK                # T = 0: nothing to do
    args = [A, 2752, A, A, A, A, A, A, A, A, A, A, A, 64, 64, None]
    for fn in (L.glmkv_mla_prep, L.glmkv_mla_prep_fp8):
        bad = list(args); bad[1] = 2748 - 64
        assert fn(*bad) == _lib.ERR_ARG                                                 # lda too small
        bad = list(args); bad[1] = 2754
        assert fn(*bad) == _lib.ERR_ALIGN                                               # lda % 4
        bad = list(args); bad[0] = A + 2
        assert fn(*bad) == _lib.ERR_ALIGN                                               # x not 8-aligned
        bad = list(args); bad[9] = None
        assert fn(*bad) == _lib.ERR_ARG                                                 # idx without ik_w
        bad = list(args); bad[13] = 32
        assert fn(*bad) == _lib.ERR_ARG                                                 # sf_rows < T
        bad = list(args); bad[14] = 0
        assert fn(*bad) == _lib.OK                                                      # T = 0
        shared = list(args); shared[1] = 2624; shared[8] = shared[9] = shared[10] = None; shared[14] = -1
        assert fn(*shared) == _lib.ERR_ARG                                              # T < 0
        # the latent cache kv needs 4-byte alignment (include/glmkv.h): 4 passes the host checks and
        # reaches the device query, which fails without a GPU (never run where a device exists: the
        # addresses are not real); 2 is rejected
        if not _has_cuda_device():
            ok4 = list(args); ok4[7] = A + 4
            assert fn(*ok4) == _lib.ERR_DEVICE
        bad = list(args); bad[7] = A + 2
        assert fn(*bad) == _lib.ERR_ALIGN
        bad = list(args); bad[8] = A + 2
        assert fn(*bad) == _lib.ERR_ALIGN                                               # idx 4-byte
    assert L.glmkv_kv_dequant(A + 8, A, 16, A, 1, A, None) == _lib.ERR_ALIGN
    assert L.glmkv_kv_dequant(A, A, 16, A, 1, A + 8, None) == _lib.ERR_ALIGN
    assert L.glmkv_kv_dequant(A, A, 16, A, -1, A, None) == _lib.ERR_ARG
    assert L.glmkv_kv_dequant(A, A, 16, A, 0, A, None) == _lib.OK
    assert L.glmkv_idx_gather(A, A, 16, A, 1, A + 4, A, None) == _lib.ERR_ALIGN
    assert L.glmkv_idx_gather(A, A, -1, A, 1, A, A, None) == _lib.ERR_ARG
    assert L.glmkv_topk_stream(A + 4, A, A, A, 8, None) == _lib.ERR_ALIGN
    assert L.glmkv_topk_slots(A, A, 16, A, A, None, 8, None) == _lib.ERR_ARG
    assert L.glmkv_mark_rows(A, A, A, -1, A, 16, None) == _lib.ERR_ARG                # T < 0
    assert L.glmkv_mark_rows(A, A, A, 8, None, 16, None) == _lib.ERR_ARG              # no mask
    assert L.glmkv_mark_rows(A, A, A, 8, A, 0, None) == _lib.ERR_ARG                  # no mask words
    assert L.glmkv_mark_rows(A, A, A, 0, A, 0, None) == _lib.OK                       # nothing at all
    assert L.glmkv_mark_rows(A, A, A, 8, A + 4, 16, None) == _lib.ERR_ALIGN           # mask 8-byte
    assert L.glmkv_mark_rows(A + 8, A, A, 8, A, 16, None) == _lib.ERR_ALIGN           # ind 16-byte
    assert L.glmkv_mark_rows(None, A, A, 8, A, 16, None) == _lib.ERR_ARG
    F = L.glmkv_topk_stream_mark  # ind, ks, klen, tlen, T, ke, mask, mask_words, stream
    assert F(A, A, A, A, -1, A, A, 16, None) == _lib.ERR_ARG                           # T < 0
    assert F(A, A, A, A, 8, A, None, 16, None) == _lib.ERR_ARG                         # no mask
    assert F(A, A, A, A, 8, A, A, 0, None) == _lib.ERR_ARG                             # no mask words
    assert F(A, A, A, A, 0, A, A, 0, None) == _lib.OK                                  # nothing at all
    assert F(A, A, None, A, 8, A, A, 16, None) == _lib.ERR_ARG                         # no klen
    assert F(A, A, A, None, 8, A, A, 16, None) == _lib.ERR_ARG                         # no tlen
    assert F(A, A, A, A, 8, None, A, 16, None) == _lib.ERR_ARG                         # no ke
    assert F(A, A, A, A, 8, A, A + 4, 16, None) == _lib.ERR_ALIGN                      # mask 8-byte
    assert F(A + 8, A, A, A, 8, A, A, 16, None) == _lib.ERR_ALIGN                      # ind 16-byte
    assert L.glmkv_kv_dequant_marked(A, A, 16, A, 0, A, A, None) == _lib.OK           # nseq = 0
    assert L.glmkv_kv_dequant_marked(A, A, 16, A, 1, None, A, None) == _lib.ERR_ARG
    assert L.glmkv_kv_dequant_marked(A, A, 16, A, 1, A + 4, A, None) == _lib.ERR_ALIGN
    assert L.glmkv_kv_dequant_marked(A + 8, A, 16, A, 1, A, A, None) == _lib.ERR_ALIGN
    with pytest.raises(glmkv.GlmKvError):
        _lib.call("glmkv_topk_stream", A + 4, A, A, A, 8, None)
    assert "misaligned" in glmkv.strerror(_lib.ERR_ALIGN)


def test_selftest_wait_rejects_bad_limits_on_the_host(built_lib):
    import glmkv
    from glmkv import _lib

    L = glmkv.lib()
    assert L.glmkv_selftest_wait(0, 0x10000, None) == _lib.ERR_ARG
    assert L.glmkv_selftest_wait(2_000_000_000, 0x10000, None) == _lib.ERR_ARG
    assert L.glmkv_selftest_wait(1000, None, None) == _lib.ERR_ARG
