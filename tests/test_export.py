"""Weight exporter (tessera-inference_b200/export_weights.py) against the
reference's tools/export_weights.py.

The golden file tests/golden/export_ref.json holds the sha256 of the .tcw the
reference's own script wrote for synth.fake_checkpoint (f32 and bf16), made by
tests/golden/make_golden.py export. Our exporter must write the same bytes,
and refuse, before writing anything, the checkpoints tc_create would reject.
"""
import hashlib
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import export_weights
import synth
import tcw

HERE = Path(__file__).resolve().parent
EXPORTER = HERE.parent / "tessera-inference_b200" / "export_weights.py"
GOLDEN = json.loads((HERE / "golden" / "export_ref.json").read_text())


def run_export(ck: Path, out: Path):
    return subprocess.run([sys.executable, str(EXPORTER), str(ck), str(out)], capture_output=True, text=True)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_export_matches_reference_bytes(tmp_path, dtype, capfd):
    ck = tmp_path / "ck.pt"
    torch.save(synth.fake_checkpoint(7, dtype), ck)
    out = tmp_path / "w.tcw"
    r = run_export(ck, out)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith(f"wrote {out}: 116 tensors, 175.3 MB")
    data = out.read_bytes()
    assert len(data) == GOLDEN[dtype]["bytes"]
    assert hashlib.sha256(data).hexdigest() == GOLDEN[dtype]["sha256"]
    assert not (tmp_path / "w.tcw.tmp").exists()
    # the widened values are the checkpoint's, exactly; the extra tensors are kept
    w = tcw.read_tcw(out)
    sd = synth.fake_checkpoint(7, dtype)["model"]
    assert list(w) == list(sd)
    for k in ("s2_backbone.embedding.0.weight", "dim_reducer.4.bias", "s2_backbone.extra_head.weight"):
        np.testing.assert_array_equal(w[k], sd[k].float().numpy())
    assert tcw.check_large({k: v.shape for k, v in w.items()}) == []
    # tc_create accepts the file: on a GPU it returns a handle; without one it
    # gets past the weights and fails at the first CUDA call
    import tessera_b200 as tb
    lib = tb.load_library()
    capfd.readouterr()
    h = lib.tc_create(str(out).encode(), 4)
    if h:
        lib.tc_destroy(h)
    else:
        err = capfd.readouterr().err
        assert err.startswith("tc_create: ") and "weights" not in err, err


def test_export_bare_state_dict_and_namespace_args():
    """A bare state dict and argparse.Namespace arguments are both accepted."""
    import argparse
    ck = synth.fake_checkpoint(7, extra=False)
    sd, args = export_weights.state_dict_of(ck["model"])
    assert sd is ck["model"] and args == {}
    sd, args = export_weights.state_dict_of({"model": ck["model"], "args": argparse.Namespace(nhead=4)})
    assert args == {"nhead": 4}
    assert export_weights.problems_of(sd, args, "ck") == []


def test_export_refuses_bad_checkpoints():
    ck = synth.fake_checkpoint(7, extra=False)
    sd, args = ck["model"], ck["args"]
    P = export_weights.problems_of
    # the reference's own argument check (tools/export_weights.py:24-28)
    assert P(sd, dict(args, nhead=8), "ck") == [
        "ck: nhead=8, but the encoder is built for nhead=4 (the v2 Large student)"]
    assert P(sd, dict(args, enable_qk_norm=True), "ck")[0].startswith("ck: enable_qk_norm=True")
    # missing tensor, wrong shape, non-finite value, non-tensor entry
    miss = dict(sd)
    del miss["s1_backbone.transformer_encoder.layers.3.linear2.bias"]
    assert P(miss, args, "ck") == ["ck: missing tensor s1_backbone.transformer_encoder.layers.3.linear2.bias"]
    bad = dict(sd, **{"dim_reducer.0.weight": torch.zeros(2560, 1279)})
    assert P(bad, args, "ck") == ["ck: dim_reducer.0.weight has shape (2560, 1279), expected (2560, 1280)"]
    nan = dict(sd)
    nan["s2_backbone.embedding.2.weight"] = sd["s2_backbone.embedding.2.weight"].clone()
    nan["s2_backbone.embedding.2.weight"][3, 4] = float("nan")
    assert P(nan, args, "ck") == ["ck: s2_backbone.embedding.2.weight holds non-finite values"]
    assert P(dict(sd, note="hello"), args, "ck") == ["ck: note is not a tensor"]
    assert P([1, 2], {}, "ck")[0].startswith("ck: no state dict found")


def test_export_cli_writes_nothing_on_error(tmp_path):
    ck = tmp_path / "small.pt"
    torch.save({"model": {"s2_backbone.embedding.0.weight": torch.zeros(640, 10)}, "args": {"nhead": 8}}, ck)
    out = tmp_path / "w.tcw"
    r = run_export(ck, out)
    assert r.returncode == 1
    assert "nhead=8, but the encoder is built for nhead=4" in r.stderr
    assert "missing tensor s2_backbone.embedding.0.bias" in r.stderr
    assert not out.exists() and not (tmp_path / "w.tcw.tmp").exists()
    r = subprocess.run([sys.executable, str(EXPORTER), str(ck)], capture_output=True, text=True)
    assert r.returncode == 1 and r.stderr.startswith("usage: python export_weights.py CHECKPOINT.pt OUT.tcw")


def test_read_tcw_rejects_truncation(tmp_path):
    p = tmp_path / "w.tcw"
    tcw.write_tcw(p, {"a": np.ones((2, 3), np.float32), "b": np.zeros(4, np.float32)})
    assert set(tcw.read_tcw(p)) == {"a", "b"}
    (tmp_path / "t.tcw").write_bytes(p.read_bytes()[:-3])
    with pytest.raises(ValueError, match="truncated"):
        tcw.read_tcw(tmp_path / "t.tcw")
    (tmp_path / "m.tcw").write_bytes(b"TCW2" + p.read_bytes()[4:])
    with pytest.raises(ValueError, match="bad weights file"):
        tcw.read_tcw(tmp_path / "m.tcw")
