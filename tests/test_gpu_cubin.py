"""The cubin a kern manifest loads (glm_glue_b200.cubin): its entries, found by the reference's names
and launched through the CUDA driver API with the launch shapes glmkv_launch_shape reports, give
the same bytes as the shared library's launchers (and so as the reference)."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES = 8
ENTRIES = ("glm_plan", "glm_mla_prep", "glm_mla_prep_fp8", "glm_idx_gather", "glm_kv_dequant", "glm_topk_stream",
           "glm_topk_slots")


class Driver:
    def __init__(self, path):
        self.cu = ctypes.CDLL("libcuda.so.1")
        self.mod = ctypes.c_void_p()
        torch.cuda.current_stream().synchronize()  # the runtime's primary context is current on this thread
        self._ok(self.cu.cuModuleLoad(ctypes.byref(self.mod), str(path).encode()), "cuModuleLoad")

    def _ok(self, rc, what):
        assert rc == 0, f"{what} failed with CUresult {rc}"

    def function(self, name):
        f = ctypes.c_void_p()
        self._ok(self.cu.cuModuleGetFunction(ctypes.byref(f), self.mod, name.encode()), f"cuModuleGetFunction {name}")
        return f

    def launch(self, name, grid, block, smem, args):
        f = self.function(name)
        if smem > 48 * 1024:
            self._ok(self.cu.cuFuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, ctypes.c_int(smem)),
                     "cuFuncSetAttribute")
        vals = [ctypes.c_uint64(a) if isinstance(a, PtrArg) else ctypes.c_int(a) for a in args]
        arr = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.byref(v), ctypes.c_void_p) for v in vals])
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        self._ok(self.cu.cuLaunchKernel(f, grid, 1, 1, block, 1, 1, smem, stream, arr, None), f"cuLaunchKernel {name}")

    def close(self):
        self.cu.cuModuleUnload(self.mod)


class PtrArg(int):
    pass


def P(t):
    return PtrArg(0 if t is None else t.data_ptr())


def test_cubin_entries_match_the_library(cuda):
    import glmkv
    from glmkv import workload as W
    from layer_case import LayerCase, to_host

    drv = Driver(glmkv.CUBIN_PATH)
    try:
        for e in ENTRIES:
            drv.function(e)
        call = W.config("cfg0", seed=6)
        case = LayerCase(call, "fp8", seed=6, with_topk=True)
        lib_d, cub_d = case.device(torch, cuda), case.device(torch, cuda)
        from layer_case import run_glmkv
        run_glmkv(case, lib_d, full=True)
        d, c, T = cub_d, call, call.T
        shape = lambda e: glmkv.launch_shape(e, T)
        g, b, s = shape("glm_plan")
        drv.launch("glm_plan", g, b, s, [P(d["cu"]), P(d["seq_lens"]), c.nseq, P(d["pos"]), P(d["ks"]), P(d["ke"]),
                                         P(d["klen"]), P(d["row_seq"]), P(d["zero"]), T])
        g, b, s = shape("glm_mla_prep_fp8")
        drv.launch("glm_mla_prep_fp8", g, b, s,
                   [P(d["x"]), case.lda, P(d["g_q"]), P(d["g_kv"]), P(d["rope"]), P(d["pos"]), P(d["slot"]), P(d["kv"]),
                    P(d["idx"]), P(d["ik_w"]), P(d["ik_b"]), P(d["qq"]), P(d["qsf"]), case.sf_rows, T])
        g, b, s = shape("glm_idx_gather")
        drv.launch("glm_idx_gather", g, b, s, [P(d["idx"]), P(d["block_table"]), c.max_pages, P(d["seq_lens"]),
                                               c.nseq, P(d["kg"]), P(d["ksf"])])
        g, b, s = shape("glm_topk_stream")
        drv.launch("glm_topk_stream", g, b, s, [P(d["ind"]), P(d["ks"]), P(d["klen"]), P(d["tlen"]), T])
        g, b, s = shape("glm_kv_dequant")
        drv.launch("glm_kv_dequant", g, b, s, [P(d["kv"]), P(d["block_table"]), c.max_pages, P(d["seq_lens"]),
                                               c.nseq, P(d["kvd"])])
        torch.cuda.synchronize()
        a, bb = to_host(lib_d, torch), to_host(cub_d, torch)
        for k in a:
            assert np.array_equal(a[k], bb[k]), k
    finally:
        drv.close()
