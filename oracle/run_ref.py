"""Run the reference's own CUDA op (oracle/_ref/dvatt_ref.so, built from its sources by
oracle/Makefile) on inputs saved with torch.save, in a process of its own (it registers
the same torch.ops.libdvatt namespace as dvattn_b200).  Test / benchmark infrastructure.

    python oracle/run_ref.py <in.pt> <out.pt> [timing_iters]

in.pt: dict(kind='paged'|'varlen', args=tuple of op arguments after `output`, out_shape,
dtype).  out.pt: dict(out=<cpu tensor>, us=<mean microseconds per call or None>).
"""
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "dvatt_ref.so")


def main():
    src, dst = sys.argv[1], sys.argv[2]
    iters = int(sys.argv[3]) if len(sys.argv) > 3 else 0
    torch.ops.load_library(LIB)
    d = torch.load(src)
    args = tuple(a.cuda() if torch.is_tensor(a) else a for a in d["args"])
    out = torch.empty(d["out_shape"], dtype=d["dtype"], device="cuda")
    op = torch.ops.libdvatt.dvattn_paged_sdpa if d["kind"] == "paged" else torch.ops.libdvatt.dvattn_varlen_paged_sdpa
    op(out, *args)
    torch.cuda.synchronize()
    us = None
    if iters:
        for _ in range(3):
            op(out, *args)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(iters):
            op(out, *args)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / iters
    torch.save(dict(out=out.cpu(), us=us), dst)


if __name__ == "__main__":
    main()
