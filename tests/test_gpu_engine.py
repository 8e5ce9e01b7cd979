"""The reference engines' MoE calls served by the B200 layer (engine adapter):
same arguments, same results as GPUStreamEngine._moe_ffn / _moe_ffn_gpu /
_moe_ffn_g4_gpu and GpuNativeEngine._moe_ffn_gpu_native, on layers loaded from
GGUF files, against the oracle restatements of those methods."""
import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import gguf, synth
from linuxnightmaresuite_b200.engine import MoEEngineAdapter
from oracle import moe_oracle as orc

from ._util import TOL_MAX_ABS, TOL_REL_L2

pytestmark = pytest.mark.gpu


def _model(tmp_path, kind):
    meta, tensors = synth.moe_gguf_tensors(kind, 3)
    path = str(tmp_path / f"{kind}.gguf")
    gguf.write_gguf(path, meta, tensors)
    p = gguf.GGUFParser(path)
    m = p.parse()
    return p, m, {n: (s, dt, raw) for n, s, dt, raw in tensors}


def _mat(t, name, e=None):
    shape, dt, raw = t[name]
    if len(shape) == 3:
        cols, rows, E = shape
        per = len(raw) // E
        raw = raw[e * per:(e + 1) * per]
    else:
        cols, rows = shape
    return orc.dequantize_matrix(np.frombuffer(raw, np.uint8), dt, rows, cols)


class _Engine:
    """Stands in for GPUStreamEngine: the methods the adapter replaces."""

    def _moe_ffn(self, xn, layer_idx, weights):
        raise AssertionError("the engine's own MoE path ran")

    def _moe_ffn_gpu(self, xn_ptr, layer_idx, weights, out_ptr=None):
        raise AssertionError("the engine's own MoE path ran")


def _check(got, exp):
    mx, rel = orc.compare(got, exp)
    assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (mx, rel)


def test_swiglu_engine_calls(tmp_path):
    p, m, t = _model(tmp_path, "swiglu")
    ad = MoEEngineAdapter(p, m, "cuda:0")
    eng = _Engine()
    ad.install(eng)
    router = np.frombuffer(t["blk.0.ffn_gate_inp.weight"][2], np.float32).reshape(16, 512)
    experts = [orc.DenseExpert(_mat(t, "blk.0.ffn_gate_exps.weight", e),
                               _mat(t, "blk.0.ffn_up_exps.weight", e),
                               _mat(t, "blk.0.ffn_down_exps.weight", e)) for e in range(16)]
    shared = orc.DenseExpert(*(_mat(t, f"blk.0.ffn_{n}_shexp.weight")
                               for n in ("gate", "up", "down")))
    rng = np.random.default_rng(4)
    for _ in range(3):
        xn = rng.standard_normal((1, 512), dtype=np.float32)
        exp, _, _ = orc.engine_moe_ffn(xn, router, experts, 4)
        exp = exp + shared.forward(xn[0])      # the file's block has a shared expert
        got = eng._moe_ffn(xn, 0, {})
        assert got.shape == (1, 512) and got.dtype == np.float32
        _check(got, exp)
        # device pointers in and out: nothing crosses to the host
        x_dev = torch.from_numpy(xn[0]).cuda()
        out_dev = torch.empty_like(x_dev)
        r = eng._moe_ffn_gpu(x_dev.data_ptr(), 0, {}, out_dev.data_ptr())
        assert r == out_dev.data_ptr()
        _check(out_dev.cpu().numpy(), exp[0])
        # in place in bufs['xn'], as GpuNativeEngine._moe_ffn_gpu_native
        bufs = {"xn": x_dev.data_ptr()}
        ad.moe_ffn_gpu_native(None, bufs, 0)
        _check(x_dev.cpu().numpy(), exp[0])
    assert ad.layer(0).device_status() == 0
    assert ad.calls == 9
    p.close()


def test_gemma4_engine_call(tmp_path):
    p, m, t = _model(tmp_path, "gemma4")
    ad = MoEEngineAdapter(p, m, "cuda:0")
    d, E, F = 512, 16, 256
    f32 = {n: np.frombuffer(raw, np.float32).reshape(tuple(s[::-1]))
           for n, (s, dt, raw) in t.items() if dt == 0}
    ds = f32["blk.0.ffn_down_exps.scale"].reshape(-1)
    _, _, gu_raw = t["blk.0.ffn_gate_up_exps.weight"]
    _, _, dn_raw = t["blk.0.ffn_down_exps.weight"]
    gper, dper = len(gu_raw) // E, len(dn_raw) // E
    experts = [orc.gemma4_expert_from_blocks(
        np.frombuffer(gu_raw[e * gper:(e + 1) * gper], np.uint8), 12,
        np.frombuffer(dn_raw[e * dper:(e + 1) * dper], np.uint8), 7, d, F, ds[e])
        for e in range(E)]
    rng = np.random.default_rng(5)
    for _ in range(3):
        attn_out = rng.standard_normal(d, dtype=np.float32) * np.float32(3)
        moe_in = orc.rms_norm(attn_out, f32["blk.0.pre_ffw_norm_2.weight"]).astype(np.float32)
        exp, _, _ = orc.gemma4_routed(attn_out, moe_in, f32["blk.0.ffn_gate_inp.weight"],
                                      f32["blk.0.ffn_gate_inp.scale"].reshape(-1), experts, 4,
                                      1e-6)
        got = ad.moe_ffn_g4_gpu(attn_out, moe_in, {}, 0, 1e-6)
        assert got.shape == (d,)
        _check(got, exp)
    p.close()
