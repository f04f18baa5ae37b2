"""Small, fixed workloads for profiling one network on one GPU.

    python -m qppocr_b200.profile_cases det   [--batch 8]  [--hw 960] [--replays 3] [--math tf32] [--table]
    python -m qppocr_b200.profile_cases rec   [--batch 32] [--replays 3]
    python -m qppocr_b200.profile_cases cls   [--batch 64]
    python -m qppocr_b200.profile_cases block

Each builds the session for its config (qppocr_b200/nets.py), runs it once
(plan, weight upload, graph capture), then replays the captured graph
`--replays` times with the inputs resident, so a profiler sees a short, known
launch sequence: the eager validation pass, the capture, then the replays.
--table prints the per-step device times (CUDA events, one eager pass per
step) with each step's algorithmic bytes and flops.
"""
import argparse
import os
import sys


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m qppocr_b200.profile_cases")
    ap.add_argument("net", choices=["det", "rec", "cls", "block"])
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--hw", type=int, default=960, help="det image side")
    ap.add_argument("--replays", type=int, default=3)
    ap.add_argument("--math", default="tf32", choices=["tf32", "3xtf32"])
    ap.add_argument("--table", action="store_true")
    a = ap.parse_args(argv)

    import qppocr_b200 as q
    from qppocr_b200 import nets

    ctx = q.CudaContext.open(int(os.environ.get("LOCAL_RANK", "0")))
    if a.net == "det":
        g, w = nets.build_det()
        x = nets.det_input(a.batch or 8, a.hw, a.hw)
        role = "det"
    elif a.net == "rec":
        g, w = nets.build_rec()
        x = nets.rec_input(a.batch or 32)
        role = "rec"
    elif a.net == "cls":
        g, w = nets.build_cls()
        x = nets.cls_input(a.batch or 64)
        role = "cls"
    else:
        g, w = nets.build_block()
        x = nets.block_input(0)
        role = "other"
    g = q.optimize(g, w)
    s = ctx.create_session(g, w, role=role, math=a.math)
    s.run({"x": x})
    ms = s.replay({"x": x}, a.replays)
    print(f"{a.net} batch {x.shape[0]} {a.math}: {ms:.3f} ms per replay", flush=True)
    if a.table:
        prof = s.profile({"x": x}, iters=3)
        for k, (kern, node, by, fl, t) in enumerate(prof):
            print(f"{k:3d} {kern:14s} {t * 1000:8.1f} us {by / 1e6:9.1f} MB {by / t / 1e6:8.0f} GB/s "
                  f"{fl / t / 1e9:7.1f} TF/s  {node}")
    s.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
