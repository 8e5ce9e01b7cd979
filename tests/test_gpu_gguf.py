"""MoE blocks loaded from GGUF files into HBM through pinned staging, against
the oracle on the same file's tensors."""
import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import _lib, gguf, synth
from oracle import moe_oracle as orc

from ._util import TOL_MAX_ABS, TOL_REL_L2, check_layer

pytestmark = pytest.mark.gpu


def _file(tmp_path, kind):
    meta, tensors = synth.moe_gguf_tensors(kind, 3)
    path = str(tmp_path / f"{kind}.gguf")
    gguf.write_gguf(path, meta, tensors)
    return path, {n: (shape, dt, raw) for n, shape, dt, raw in tensors}


def _mat(t, name, e=None):
    shape, dt, raw = t[name]
    if len(shape) == 3:
        cols, rows, E = shape
        per = len(raw) // E
        raw = raw[e * per:(e + 1) * per]
    else:
        cols, rows = shape
    return orc.dequantize_matrix(np.frombuffer(raw, np.uint8), dt, rows, cols)


def test_swiglu_block_from_file_matches_oracle(tmp_path):
    path, t = _file(tmp_path, "swiglu")
    with gguf.GGUFParser(path) as p:
        m = p.parse()
        stager = gguf.PinnedStager("cuda:0", chunk_bytes=1 << 20)
        layer = gguf.load_moe_layer(p, m, 0, "cuda:0", stager=stager)
        assert stager.bytes_moved == sum(len(raw) for n, (s, d, raw) in t.items()
                                         if "_exps" in n or "_shexp" in n)
    router = np.frombuffer(t["blk.0.ffn_gate_inp.weight"][2], np.float32).reshape(16, 512)
    experts = [orc.DenseExpert(_mat(t, "blk.0.ffn_gate_exps.weight", e),
                               _mat(t, "blk.0.ffn_up_exps.weight", e),
                               _mat(t, "blk.0.ffn_down_exps.weight", e)) for e in range(16)]
    shared = orc.DenseExpert(*(_mat(t, f"blk.0.ffn_{n}_shexp.weight") for n in ("gate", "up",
                                                                                  "down")))
    x = np.random.default_rng(1).standard_normal((20, 512), dtype=np.float32)
    out, ids, w = layer.forward_batch(torch.from_numpy(x).cuda(), return_routing=True)
    torch.cuda.synchronize()
    assert layer.device_status() == 0
    check_layer(x, np.ascontiguousarray(router.T), None, 4, 1, experts, shared,
                out.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy())


def test_gemma4_block_from_file_matches_oracle(tmp_path):
    path, t = _file(tmp_path, "gemma4")
    with gguf.GGUFParser(path) as p:
        m = p.parse()
        block = gguf.load_moe_layer(p, m, 0, "cuda:0")
    d, E, F = 512, 16, 256
    f32 = {n: np.frombuffer(raw, np.float32).reshape(tuple(s[::-1]))
           for n, (s, dt, raw) in t.items() if dt == 0}
    ds = f32["blk.0.ffn_down_exps.scale"].reshape(-1)
    gu_shape, _, gu_raw = t["blk.0.ffn_gate_up_exps.weight"]
    dn_shape, _, dn_raw = t["blk.0.ffn_down_exps.weight"]
    gper, dper = len(gu_raw) // E, len(dn_raw) // E
    experts = [orc.gemma4_expert_from_blocks(np.frombuffer(gu_raw[e * gper:(e + 1) * gper], np.uint8),
                                             12, np.frombuffer(dn_raw[e * dper:(e + 1) * dper],
                                                               np.uint8), 7, d, F, ds[e])
               for e in range(E)]
    w = {"moe_router": f32["blk.0.ffn_gate_inp.weight"],
         "moe_gate_inp_scale": f32["blk.0.ffn_gate_inp.scale"].reshape(-1),
         "ffn_norm": f32["blk.0.ffn_norm.weight"],
         "wg": _mat(t, "blk.0.ffn_gate.weight"), "wu": _mat(t, "blk.0.ffn_up.weight"),
         "wd": _mat(t, "blk.0.ffn_down.weight"),
         "post_ffw_norm_1": f32["blk.0.post_ffw_norm_1.weight"],
         "pre_ffw_norm_2": f32["blk.0.pre_ffw_norm_2.weight"],
         "post_ffw_norm_2": f32["blk.0.post_ffw_norm_2.weight"]}
    x = np.random.default_rng(2).standard_normal((9, d), dtype=np.float32) * np.float32(3)
    got = block.forward(x)
    assert block.device_status() == 0
    for r in range(9):
        exp, _, _ = orc.gemma4_moe_block(x[r], w, experts, 4, 1e-6)
        mx, rel = orc.compare(got[r], exp)
        assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (r, mx, rel)


def test_expert_subset_upload_is_bit_exact(tmp_path):
    path, t = _file(tmp_path, "swiglu")
    name = "blk.0.ffn_down_exps.weight"
    shape, dt, raw = t[name]
    per = len(raw) // shape[2]
    with gguf.GGUFParser(path) as p:
        m = p.parse()
        stager = gguf.PinnedStager("cuda:0", chunk_bytes=4096, n_buffers=3)
        sel = [4, 5, 6, 9, 15]
        got, sl = gguf.upload_experts(p, m, name, sel, stager)
        stager.finish()
    assert got.shape == (5, shape[1], per // shape[1])
    host = got.cpu().numpy().reshape(5, -1)
    for i, e in enumerate(sel):
        assert host[i].tobytes() == raw[e * per:(e + 1) * per]
