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
           "glm_topk_slots", "glm_q_post", "glm_add_rms_quant", "glm_quant", "glm_mqa_logits_paged")


class TensorMap(ctypes.Structure):
    """CUtensorMap: 128 opaque bytes, 64-byte aligned, passed to a kernel by value."""
    _align_ = 64
    _fields_ = [("opaque", ctypes.c_uint64 * 16)]


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
        vals = [a if isinstance(a, TensorMap) else ctypes.c_uint64(a) if isinstance(a, PtrArg) else ctypes.c_int(a)
                for a in args]
        arr = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.byref(v), ctypes.c_void_p) for v in vals])
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        self._ok(self.cu.cuLaunchKernel(f, grid, 1, 1, block, 1, 1, smem, stream, arr, None), f"cuLaunchKernel {name}")

    def tensor_map_u8(self, base, dims, strides, box):
        """A tiled u8 tensor map with the 128-byte swizzle and 256-byte L2 promotion, as the library's
        launcher of glm_mqa_logits_paged encodes it (csrc/glmkv.cu)."""
        tm = TensorMap()
        n = len(dims)
        u64, u32 = ctypes.c_uint64, ctypes.c_uint32
        rc = self.cu.cuTensorMapEncodeTiled(ctypes.byref(tm), 0, n, ctypes.c_void_p(base), (u64 * n)(*dims),
                                            (u64 * (n - 1))(*strides), (u32 * n)(*box), (u32 * n)(*([1] * n)), 0, 3, 3,
                                            0)
        self._ok(rc, "cuTensorMapEncodeTiled")
        return tm

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


def test_cubin_mqa_logits_matches_the_library(cuda):
    """glm_mqa_logits_paged from the cubin, with tensor maps encoded through the driver API as a kern
    manifest would and the launch shape glmkv_launch_shape reports: the same logits as
    the library's launcher."""
    import glmkv
    from glmkv import workload as W

    rng = np.random.default_rng(91)
    call = W.make_call([300, 0, 70], [40, 21, 9], rng, spare_pages=3)
    codes = rng.integers(0, 256, size=call.n_pages * 64 * 132, dtype=np.uint8)
    codes = np.where((codes & 0x7F) == 0x7F, codes - 1, codes).astype(np.uint8)
    pool = codes.reshape(call.n_pages, 64 * 132)
    pool[:, 8192:] = np.exp2(rng.integers(-8, 4, size=(call.n_pages, 64))).astype(np.float32).view(np.uint8)
    R = call.T
    iq = rng.integers(0, 126, size=R * 32 * 128, dtype=np.uint8)
    w = rng.standard_normal((R, 32)).astype(np.float32)
    row_seq = np.repeat(np.arange(call.nseq, dtype=np.int32), call.fresh)
    klen = (W.positions(call) + 1).astype(np.int32)
    stride = int(klen.max())
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    iq_d, pool_d, bt_d, rs_d, kl_d, w_d = t(iq), t(pool.reshape(-1)), t(call.block_table), t(row_seq), t(klen), t(w)
    outs = []
    drv = Driver(glmkv.CUBIN_PATH)
    try:
        for via in ("lib", "cubin"):
            logits = torch.full((R * stride,), float("nan"), dtype=torch.float32, device=cuda)
            if via == "lib":
                glmkv.mqa_logits_paged(iq_d, pool_d, call.n_pages, bt_d, call.max_pages, rs_d, kl_d, w_d, logits,
                                       stride, R)
            else:
                tm_q = drv.tensor_map_u8(iq_d.data_ptr(), [128, R * 32], [128], [128, 256])
                tm_k = drv.tensor_map_u8(pool_d.data_ptr(), [128, 64, call.n_pages], [128, 8448], [128, 64, 1])
                g, b, sm = glmkv.launch_shape("glm_mqa_logits_paged", R)
                drv.launch("glm_mqa_logits_paged", g, b, sm,
                           [tm_q, tm_k, P(pool_d), call.n_pages, P(bt_d), call.max_pages, P(rs_d), P(kl_d), P(w_d),
                            P(logits), stride, R])
            torch.cuda.synchronize()
            outs.append(logits.cpu().numpy())
    finally:
        drv.close()
    assert glmkv.fault_flags() == 0
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    assert np.isfinite(outs[0].reshape(R, stride)[0, :klen[0]]).all()


def _snippet_shapes():
    """(entry, grid expression, block, dynamic shared memory) of every launch in INTEGRATION.md's
    manifest snippets."""
    import pathlib
    import re

    text = (pathlib.Path(__file__).resolve().parents[1] / "INTEGRATION.md").read_text()
    out = []
    # G.b200(entry, params, grid, block[, smem]): params a name or a list expression, possibly over lines
    # (never reaching into the next call); the grid's first element may hold one level of brackets
    params = r'((?:(?!G\.b200\().)*?)'
    shape = r'\[((?:[^\[\]]|\[[^\[\]]*\])+?), 1, 1\],\s*\[(\d+), 1, 1\](?:,\s*(\d+))?'
    for m in re.finditer(r'G\.b200\((?:"(glm_\w+)"|prep),' + params + shape, text, flags=re.S):
        entries = [m.group(1)] if m.group(1) else ["glm_mla_prep_fp8", "glm_mla_prep"]
        for e in entries:
            out.append((e, m.group(3), int(m.group(4)), int(m.group(5) or 0)))
    for m in re.finditer(r'launch\("glm_glue_b200", "(glm_\w+)", \[(.+?), 1, 1\], \[(\d+), 1, 1\],\s*(\d+)', text):
        out.append((m.group(1), m.group(2), int(m.group(3)), int(m.group(4))))
    return out


def test_integration_snippet_matches_the_launch_shapes(cuda):
    """Every launch of INTEGRATION.md's manifest snippets uses the block and dynamic shared memory the
    library launches that entry with, and (with the device's SM count for SMS_B200 and T = 16,384) its
    grid. A snippet that gave a kernel less shared memory than it uses would corrupt its results."""
    import re

    import glmkv

    T = 16384
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    shapes = _snippet_shapes()
    assert {e for e, *_ in shapes} == set(ENTRIES) | {"glm_mark_rows", "glm_kv_dequant_marked", "glm_topk_stream_mark"}, \
        sorted({e for e, *_ in shapes})

    def grid_of(expr):
        expr = expr.strip().replace("G.SMS_B200", "SMS").replace("SMS_B200", "SMS")
        m = re.fullmatch(r'\{"ceil_div": \[(\w+), (\d+)\]\}', expr)
        if m:
            return -(-{"T": T}[m.group(1)] // int(m.group(2)))
        return eval(expr, {"SMS": sms, "T": T})

    for entry, grid, block, smem in shapes:
        if entry == "glm_quant":  # its grid depends on K as well: block 256, no shared memory
            assert (block, smem) == (256, 0), entry
            continue
        g, b, s = glmkv.launch_shape(entry, T)
        assert (block, smem) == (b, s), f"{entry}: snippet block {block} smem {smem}, library {b} {s}"
        assert grid_of(grid) == g, f"{entry}: snippet grid {grid} = {grid_of(grid)}, library {g}"
