"""Time one back-end kernel alone on a synthetic chunk, through the library's
operator entry points (include/tessera_b200_ops.h), with CUDA events.

  python tessera-inference_b200/op_bench.py attention --T 120        # uniform series of 120 steps
  python tessera-inference_b200/op_bench.py layernorm --M 131072

Prints one JSON line: microseconds per launch, the algorithmic bytes of the
launch and the bandwidth they give. Attention bytes per token are the Q, K and
V rows read (3 x 640 bf16) and the output row written (640 bf16): 5,120 B.
LayerNorm bytes per row are 640 bf16 read and written: 2,560 B. Inputs are
seeded random bf16 in device memory, larger than L2 at the default sizes.
`TC_ATTN_TC=2` selects the tcgen05 attention kernel for every series of up
to 128 steps and `TC_ATTN_TC=0` the mma.sync kernel; unset, the library
takes tcgen05 for series longer than 48 steps and up to 128.

The chunk is described by its series length alone (no offsets array), so the
entry point does no host work and the launches run back to back.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
import tessera_b200 as tb  # noqa: E402


def time_launches(fn, reps: int) -> float:
    """Microseconds per launch over `reps` launches after three warm-up ones."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / reps


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("op", choices=["attention", "layernorm"])
    ap.add_argument("--T", type=int, default=120, help="uniform series length (attention)")
    ap.add_argument("--tokens", type=int, default=131072, help="tokens per attention chunk")
    ap.add_argument("--M", type=int, default=131072, help="rows (layernorm)")
    ap.add_argument("--reps", type=int, default=10)
    a = ap.parse_args(argv)
    lib = tb.load_library()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(0)
    if a.op == "attention":
        npix = a.tokens // a.T
        M = npix * a.T
        qkv = torch.randn(M, 1920, device="cuda", generator=g).to(torch.bfloat16)
        att = torch.empty(M, 640, device="cuda", dtype=torch.bfloat16)

        def run():
            if lib.tcb_op_attention(qkv.data_ptr(), None, a.T, npix, a.T, att.data_ptr(), st):
                raise RuntimeError("tcb_op_attention failed")

        us = time_launches(run, a.reps)
        nbytes = M * 5120
        rec = {"op": "attention", "tokens": M, "pixels": npix, "T": a.T}
    else:
        M = a.M
        x = torch.randn(M, 640, device="cuda", generator=g).to(torch.bfloat16)
        y = torch.empty_like(x)
        gam = torch.ones(640, device="cuda")
        bet = torch.zeros(640, device="cuda")

        def run():
            if lib.tcb_op_layernorm640(x.data_ptr(), M, gam.data_ptr(), bet.data_ptr(), y.data_ptr(), st):
                raise RuntimeError("tcb_op_layernorm640 failed")

        us = time_launches(run, a.reps)
        nbytes = M * 2560
        rec = {"op": "layernorm640", "rows": M}
    rec.update({"us_per_launch": round(us, 2), "bytes_per_launch": nbytes, "GB_per_s": round(nbytes / us / 1e3, 1),
                "reps": a.reps})
    print(json.dumps(rec))
    return 0


if __name__ == "__main__":
    sys.exit(main())
