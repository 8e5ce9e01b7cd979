"""GGUF reading against the reference's own parser (gguf_parser.py), and the
expert-slice arithmetic (nightmare_stream.py:3361-3441).  CPU only."""
import hashlib
import json
import os

import numpy as np
import pytest

from linuxnightmaresuite_b200 import gguf, synth

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module", params=["swiglu", "gemma4"])
def model_file(request, tmp_path_factory):
    kind = request.param
    meta, tensors = synth.moe_gguf_tensors(kind, 3)
    path = str(tmp_path_factory.mktemp("gguf") / f"{kind}.gguf")
    gguf.write_gguf(path, meta, tensors)
    return kind, path, meta, tensors


def _golden(kind):
    z = np.load(os.path.join(GOLD, "gguf.npz"))
    return json.loads(str(z[f"{kind}_json"])), z


def test_writer_reproduces_the_file_the_reference_parsed(model_file):
    kind, path, _, _ = model_file
    rec, _ = _golden(kind)
    with open(path, "rb") as f:
        assert hashlib.sha256(f.read()).hexdigest() == rec["file_sha"]


def test_parse_matches_reference_parser(model_file):
    kind, path, meta, tensors = model_file
    rec, z = _golden(kind)
    with gguf.GGUFParser(path) as p:
        m = p.parse()
        assert m.version == rec["version"]
        assert m.tensor_data_offset == rec["tensor_data_offset"]
        assert json.loads(json.dumps(m.metadata, sort_keys=True)) == rec["metadata"]
        infos = {n: [list(i.shape), i.dtype, i.offset] for n, i in m.tensors.items()}
        assert infos == rec["infos"]
        for n in m.tensors:
            raw, dt, shape, ne = p.load_tensor_raw(m, n)
            assert [hashlib.sha256(raw.tobytes()).hexdigest(), ne] == rec["raw_sha"][n], n
            if dt == 0:
                assert np.array_equal(p.load_f32(m, n), z[f"{kind}_f32_{n}"]), n
        assert m.expert_count == 16 and m.expert_used_count == 4
        assert m.architecture == ("gemma4" if kind == "gemma4" else "qwen3moe")


def test_expert_slices_are_the_experts_rows(model_file):
    kind, path, _, tensors = model_file
    by_name = {n: (shape, dt, raw) for n, shape, dt, raw in tensors}
    with gguf.GGUFParser(path) as p:
        m = p.parse()
        for name in [n for n in m.tensors if n.endswith("_exps.weight")]:
            shape, dt, raw = by_name[name]
            sl = gguf.expert_slices(m, name)
            assert len(sl) == shape[2]
            per = len(raw) // shape[2]
            for e in (0, 5, shape[2] - 1):
                got = bytes(p.view(m, sl[e].offset, sl[e].nbytes))
                assert got == raw[e * per:(e + 1) * per], (name, e)
                assert (sl[e].rows, sl[e].cols, sl[e].dtype) == (shape[1], shape[0], dt)


def test_rejects_non_gguf(tmp_path):
    bad = tmp_path / "x.gguf"
    bad.write_bytes(b"NOTGGUF" + b"\0" * 64)
    with pytest.raises(ValueError):
        gguf.GGUFParser(str(bad)).parse()
