"""Convert a Tessera v2 pixel-student checkpoint to the .tcw file that tc_create reads.

usage: python export_weights.py CHECKPOINT.pt OUT.tcw

Same command line, inputs and output bytes as the reference's
tools/export_weights.py:1-40:

* the checkpoint is a dict holding the state dict under "model" (and the
  training arguments under "args"), or a bare state dict (:20-21);
* the arguments, where present, must name the Large student's sizes (:24-28);
* every tensor is written in the state dict's order as f32, so a bf16 or f16
  checkpoint is widened exactly (:22, :31-39).

Checks the reference's script leaves to the loader, made here before anything
is written so that a bad checkpoint never yields a .tcw:

* every tensor the back end reads is present with its shape (the list of
  tc_create's validation);
* those tensors hold only finite values;
* every state-dict entry is a tensor.

The file is written to OUT.tcw.tmp and renamed, so an interrupted export leaves
no partial OUT.tcw. Extra tensors (other heads, buffers) are kept, as the
reference keeps them; the back ends ignore them.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
from tcw import check_large, weight_shapes, write_tcw  # noqa: E402

# Model sizes the encoder is built for (tools/export_weights.py:25-26).
EXPECT_ARGS = {"latent_dim": 160, "num_layers": 4, "nhead": 4, "dim_feedforward": 2560, "repr_dim": 128,
               "enable_qk_norm": False}


def state_dict_of(payload):
    """The state dict and the training arguments (a dict, possibly empty)."""
    sd = payload["model"] if isinstance(payload, dict) and "model" in payload else payload
    args = payload.get("args", {}) if isinstance(payload, dict) else {}
    if args is None:
        args = {}
    if not isinstance(args, dict):  # an argparse.Namespace saved with the checkpoint
        args = vars(args)
    return sd, args


def problems_of(sd, args, src: str) -> list[str]:
    out = []
    for k, v in EXPECT_ARGS.items():
        if k in args and type(v)(args[k]) != v:
            out.append(f"{src}: {k}={args[k]}, but the encoder is built for {k}={v} (the v2 Large student)")
    if not hasattr(sd, "items"):
        return out + [f"{src}: no state dict found (expected a dict of tensors or a dict with a 'model' entry)"]
    import torch
    bad = [k for k, v in sd.items() if not isinstance(v, torch.Tensor)]
    out += [f"{src}: {k} is not a tensor" for k in bad]
    shapes = {k: tuple(v.shape) for k, v in sd.items() if isinstance(v, torch.Tensor)}
    out += [f"{src}: {p}" for p in check_large(shapes)]
    if not out:
        for name, _ in weight_shapes():
            if not bool(torch.isfinite(sd[name].detach().float()).all()):
                out.append(f"{src}: {name} holds non-finite values")
    return out


def export(src: str, out: str) -> int:
    import torch
    payload = torch.load(src, map_location="cpu", weights_only=False)
    sd, args = state_dict_of(payload)
    problems = problems_of(sd, args, src)
    if problems:
        for p in problems:
            print(p, file=sys.stderr)
        return 1
    arrays = {k: v.detach().float().contiguous().numpy() for k, v in sd.items()}
    tmp = out + ".tmp"
    try:
        write_tcw(tmp, arrays)
        os.replace(tmp, out)
    finally:
        if os.path.exists(tmp):
            os.remove(tmp)
    print(f"wrote {out}: {len(arrays)} tensors, {os.path.getsize(out) / 1e6:.1f} MB")
    return 0


def main(argv: list[str]) -> int:
    if len(argv) != 3:
        print(__doc__.strip().splitlines()[2], file=sys.stderr)
        return 1
    return export(argv[1], argv[2])


if __name__ == "__main__":
    sys.exit(main(sys.argv))
