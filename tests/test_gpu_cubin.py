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
           "glm_topk_slots", "glm_q_post", "glm_add_rms_quant", "glm_quant")


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
        if smem > 0:  # dynamic plus static shared memory above 48 KB needs the opt-in
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


def test_cubin_glue_entries_match_the_library(cuda):
    """glm_q_post, glm_add_rms_quant and glm_quant from the cubin, launched through the driver API,
    against the library's launchers on the same inputs."""
    import glmkv
    from layer_case import LDB, norm_case, q_post_case, quant_case

    drv = Driver(glmkv.CUBIN_PATH)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    try:
        T = 300
        c = q_post_case(T, 71)
        qb, rope, pos, iw = t(c["qb"].view(np.int16)), t(c["rope"].view(np.int16)), t(c["pos"]), t(c["iw"].view(np.int16))
        for full in (1, 0):
            outs = []
            for via in ("lib", "cubin"):
                qmla = torch.zeros(T * 64 * 576, dtype=torch.int16, device=cuda)
                iq = torch.zeros(T * 32 * 128, dtype=torch.uint8, device=cuda)
                wout = torch.zeros(T * 32, dtype=torch.float32, device=cuda)
                args = [P(qb), LDB, P(rope), P(pos), P(qmla), P(iq if full else None), P(iw if full else None),
                        P(wout if full else None), full, T]
                if via == "lib":
                    glmkv.q_post_full(*[a if not isinstance(a, PtrArg) else int(a) for a in args])
                else:
                    g, b, sm = glmkv.launch_shape("glm_q_post", T)
                    drv.launch("glm_q_post", g, b, sm, args)
                torch.cuda.synchronize()
                outs.append([x.cpu().numpy().view(np.uint8) for x in (qmla, iq, wout)])
            for x, y in zip(*outs):
                assert np.array_equal(x, y), f"q_post full={full}"

        a_, res_, gamma = norm_case(64, 72, True)
        for with_a in (True, False):
            outs = []
            for via in ("lib", "cubin"):
                res = t(res_.view(np.int16))
                normed = torch.zeros(64 * 6144, dtype=torch.int16, device=cuda)
                q = torch.zeros(64 * 6144, dtype=torch.uint8, device=cuda)
                sf = torch.zeros(12 * 64 * 4, dtype=torch.uint8, device=cuda)
                args = [P(t(a_.view(np.int16)) if with_a else None), P(res), P(t(gamma.view(np.int16))), P(normed), P(q),
                        P(sf), 64, 64]
                if via == "lib":
                    glmkv.add_rms_quant(*[int(a) if isinstance(a, PtrArg) else a for a in args])
                else:
                    g, b, sm = glmkv.launch_shape("glm_add_rms_quant", 64)
                    drv.launch("glm_add_rms_quant", g, b, sm, args)
                torch.cuda.synchronize()
                outs.append([x.cpu().numpy().view(np.uint8) for x in (res, normed, q, sf)])
            for x, y in zip(*outs):
                assert np.array_equal(x, y), f"add_rms_quant with_a={with_a}"

        T, K, ldx = 37, 640, 648
        x = t(quant_case(T, K, ldx).view(np.int16))
        outs = []
        for via in ("lib", "cubin"):
            q = torch.zeros(T * K, dtype=torch.uint8, device=cuda)
            sf = torch.zeros((K + 511) // 512 * T * 4, dtype=torch.uint8, device=cuda)
            args = [P(x), ldx, P(q), P(sf), T, K, T]
            if via == "lib":
                glmkv.quant_o(*[int(a) if isinstance(a, PtrArg) else a for a in args])
            else:  # grid ceil(T * ceil(K / 512) / 8), block 256 (glmkv_launch_shape cannot give it without K)
                drv.launch("glm_quant", (T * ((K + 511) // 512) + 7) // 8, 256, 0, args)
            torch.cuda.synchronize()
            outs.append([y.cpu().numpy() for y in (q, sf)])
        for a, b in zip(*outs):
            assert np.array_equal(a, b), "quant"
    finally:
        drv.close()
