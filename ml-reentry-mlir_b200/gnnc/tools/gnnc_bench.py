"""gnnc-bench: compile a model, execute it, compare to torch eager (and time it).

    python -m gnnc.tools.gnnc_bench --model gcn
    python -m gnnc.tools.gnnc_bench --model gat --dataset c2
    python -m gnnc.tools.gnnc_bench --model gat --dataset c3 --dtype bf16 --time
    python -m gnnc.tools.gnnc_bench --model gat --dataset c4 --gpus 8 --time --no-check

Same flow and exit codes as the reference's gnnc/tools/gnnc_bench.py:29-85:
0 = PASS, 1 = output mismatch, 2 = ValueError / NotImplementedError,
3 = ImportError (missing library). Differences: the default --target is b200
(the MLIR cpu/gpu targets are not part of this build and exit 3), --dataset
also accepts the synthetic workloads c1..c5, the comparison tolerance follows
the feature dtype (rtol 1e-3 / atol 1e-4 for fp32 as in the reference; 2e-2
for bf16 features), --time reports CUDA-event medians per forward, and
--gpus P runs the row-partitioned forward of gnnc.b200.distributed on P GPUs
(relaunching itself under torch.distributed.run, one process per GPU).
"""

from __future__ import annotations

import argparse
import sys

import numpy as np

from gnnc import __version__, paths
from gnnc.examples import MODELS_DIR, available


def _time_forward(lowered, inputs, warmup: int, iters: int) -> dict:
    """CUDA-event timing of the device-resident forward (graph already on the
    device), plus per-layer projection / aggregation times and edges/s."""
    import torch

    x, graph = inputs
    dev = lowered.device
    xd = x.to(dev)
    gd = graph.to(dev)
    for _ in range(warmup):
        lowered.run_device(xd, gd)
    torch.cuda.synchronize(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    for i in range(iters):
        starts[i].record()
        lowered.run_device(xd, gd)
        stops[i].record()
    torch.cuda.synchronize(dev)
    ms = sorted(s.elapsed_time(e) for s, e in zip(starts, stops, strict=True))
    # per-layer breakdown (separate, event-instrumented passes)
    per = None
    for _ in range(max(3, iters // 10)):
        evs: list = []
        lowered.run_device(xd, gd, events=evs)
        torch.cuda.synchronize(dev)
        cur = [(a.elapsed_time(b), b.elapsed_time(c)) for a, b, c in evs]
        per = cur if per is None else [(min(p0, c0), min(p1, c1)) for (p0, p1), (c0, c1) in zip(per, cur)]
    # the same forward replayed from a captured CUDA graph (small graphs)
    graph_ms = None
    if lowered._replay(xd, gd) is not None:
        for _ in range(warmup):
            lowered._replay(xd, gd)
        torch.cuda.synchronize(dev)
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(iters):
            lowered._replay(xd, gd)
        e0.record()
        torch.cuda.synchronize(dev)
        graph_ms = s0.elapsed_time(e0) / iters
    edges = lowered.graph_edges(gd, x.size(0))
    layers = [
        {"layer": i + 1, "proj_ms": pj, "agg_ms": ag, "edges": e, "agg_edges_per_s": e / (ag / 1e3),
         "nodes_per_s": x.size(0) / ((pj + ag) / 1e3)}
        for i, ((pj, ag), e) in enumerate(zip(per, edges))
    ]
    return {"median_ms": ms[len(ms) // 2], "p90_ms": ms[int(len(ms) * 0.9)], "iters": iters,
            "cuda_graph_ms": graph_ms, "layers": layers}


def _relaunch(argv: list[str], gpus: int) -> int:
    """Runs this command again under torch.distributed.run, one process per GPU."""
    import socket
    import subprocess

    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={gpus}", "--master-addr", "127.0.0.1", f"--master-port={port}",
           "-m", "gnnc.tools.gnnc_bench", *argv]
    return subprocess.call(cmd)


def _main_distributed(args) -> int:
    """--gpus P under torchrun: row-partitioned forward (gnnc.b200.distributed)."""
    import os
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from gnnc.b200 import partition as P
    from gnnc.b200.distributed import distribute
    from gnnc.compile import compile_executable
    from gnnc.ingress import get_model_and_data

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    say = print if rank == 0 else (lambda *a, **k: None)
    try:
        model, inputs = get_model_and_data(MODELS_DIR / f"{args.model}.py", args.dataset)
        model.eval()
        if args.dtype == "bf16" and inputs[0].dtype != torch.bfloat16:
            inputs = (inputs[0].to(torch.bfloat16), *inputs[1:])
        x, graph = inputs
        exe, _ = compile_executable(model, inputs, target=args.target, dtype=args.dtype,
                                    device=dev)
        dexe = distribute(exe)
        rr = P.row_range(x.size(0), world, rank)
        out = dexe.run_device(x[rr.begin : rr.end].to(dev), graph)
        # every rank's rows, padded to R, gathered on the device
        R = rr.rows_per_rank
        pad = torch.zeros((R, out.size(1)), dtype=out.dtype, device=dev)
        pad[: rr.count] = out
        full = torch.empty((world * R, out.size(1)), dtype=out.dtype, device=dev)
        dist.all_gather_into_tensor(full, pad)
        actual = full[: x.size(0)].float().cpu().numpy()
        say(f"  gpus     : {world} (rows partitioned, exchanges {dexe.exchange_modes()})")
        if args.time:
            xd = x[rr.begin : rr.end].to(dev)
            for _ in range(args.warmup):
                dexe.run_device(xd, graph)
            torch.cuda.synchronize(dev)
            dist.barrier()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.iters):
                dexe.run_device(xd, graph)
            e.record()
            torch.cuda.synchronize(dev)
            t = torch.tensor([s.elapsed_time(e) / args.iters], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            say(f"  forward  : {float(t):.3f} ms (mean of {args.iters}, max over ranks)")
            # the same forwards as one pipelined stream of batches
            dist.barrier()
            s.record()
            for _ in dexe.run_stream((xd for _ in range(args.iters)), graph):
                pass
            e.record()
            torch.cuda.synchronize(dev)
            ts = torch.tensor([s.elapsed_time(e) / args.iters], dtype=torch.float64, device=dev)
            dist.all_reduce(ts, op=dist.ReduceOp.MAX)
            say(f"  stream   : {float(ts):.3f} ms per batch (run_stream: the first layer's "
                "exchange of batch k+1 overlaps batch k)")
            if args.json and rank == 0:
                import json

                print(json.dumps({"model": args.model, "dataset": args.dataset, "gpus": world,
                                  "forward_ms": float(t), "stream_ms_per_batch": float(ts)}))
        dist.barrier()
        dexe.close()
        code = 0
        if rank == 0 and not args.no_check:
            with torch.no_grad():
                ref = model(x.to(torch.float32), graph).cpu().numpy()
            max_abs = float(np.abs(actual - ref).max())
            say(f"  out shape: {actual.shape}, max abs diff vs torch: {max_abs:.3e}")
            bf16 = exe.program.feature_dtype == torch.bfloat16
            rtol, atol = (2e-2, 2e-2) if bf16 else (1e-3, 1e-4)
            try:
                np.testing.assert_allclose(actual, ref, rtol=rtol, atol=atol)
                say("PASS")
            except AssertionError as exc:
                say("FAIL")
                say(exc)
                code = 1
        elif rank == 0:
            say(f"  out shape: {actual.shape} (not checked)")
    finally:
        dist.destroy_process_group()
    return code


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(
        prog="gnnc-bench", description="Compile a model and compare its output to torch eager."
    )
    parser.add_argument("--model", required=True, choices=available())
    parser.add_argument("--dataset", "--config", default=None,
                        help="cora | ogbn-arxiv | ogbn-products | c1 | c2 | c3 | c3-bf16 | c4; omit for get_inputs()")
    parser.add_argument("--gpus", type=int, default=1,
                        help="P > 1: row-partitioned forward on P GPUs (one process each)")
    parser.add_argument("--target", default="b200", choices=("b200", "cpu", "gpu"))
    parser.add_argument("--dtype", default=None, choices=("fp32", "bf16"),
                        help="feature dtype on the device (default: the input's)")
    parser.add_argument("--no-check", action="store_true", help="skip the eager comparison")
    parser.add_argument("--time", action="store_true", help="time the forward with CUDA events")
    parser.add_argument("--warmup", type=int, default=20)
    parser.add_argument("--iters", type=int, default=100)
    parser.add_argument("--json", action="store_true", help="also print the timing as one JSON line")
    args = parser.parse_args(argv)
    if args.gpus > 1:
        import os

        if "RANK" not in os.environ:
            return _relaunch(list(sys.argv[1:] if argv is None else argv), args.gpus)
        if int(os.environ.get("RANK", "0")) == 0:
            print(f"gnnc-bench {__version__}")
            print(f"  model    : {args.model}")
            print(f"  dataset  : {args.dataset or '<synthetic>'}")
            print(f"  target   : {args.target}")
        try:
            return _main_distributed(args)
        except ImportError as exc:
            print(f"error: {exc}", file=sys.stderr)
            return 3
        except (ValueError, NotImplementedError) as exc:
            print(f"error: {exc}", file=sys.stderr)
            return 2

    print(f"gnnc-bench {__version__}")
    print(f"  model    : {args.model}")
    print(f"  dataset  : {args.dataset or '<synthetic>'}")
    print(f"  target   : {args.target}")
    print(f"  DATA_DIR : {paths.DATA_DIR}")

    try:
        import torch

        from gnnc.compile import compile_executable
        from gnnc.execution import run_jit
        from gnnc.ingress import get_model_and_data

        model, forward_inputs = get_model_and_data(MODELS_DIR / f"{args.model}.py", args.dataset)
        model.eval()
        if args.dtype == "bf16" and forward_inputs[0].dtype != torch.bfloat16:
            forward_inputs = (forward_inputs[0].to(torch.bfloat16), *forward_inputs[1:])
        lowered, results = compile_executable(model, forward_inputs, target=args.target,
                                              dtype=args.dtype)
        outs = run_jit(lowered, results, forward_inputs)
        ref = None
        if not args.no_check:
            with torch.no_grad():
                x = forward_inputs[0]
                eager_inputs = (x.to(torch.float32), *forward_inputs[1:])
                ref = model(*eager_inputs).cpu().numpy()
        timing = _time_forward(lowered, forward_inputs, args.warmup, args.iters) if args.time else None
    except ImportError as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 3
    except (ValueError, NotImplementedError) as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 2

    if len(outs) != 1:
        print(f"error: multi-output models not yet supported (got {len(outs)})", file=sys.stderr)
        return 2
    actual = outs[0].cpu().numpy()
    if timing:
        print(f"  forward  : median {timing['median_ms']:.3f} ms, p90 {timing['p90_ms']:.3f} ms")
        if timing["cuda_graph_ms"] is not None:
            print(f"  forward  : {timing['cuda_graph_ms']:.3f} ms replayed from a CUDA graph (mean)")
        for lay in timing["layers"]:
            print(f"  layer {lay['layer']}  : proj {lay['proj_ms']:.3f} ms, agg {lay['agg_ms']:.3f} ms, "
                  f"{lay['edges']} edges, {lay['agg_edges_per_s'] / 1e9:.2f} G edges/s (agg), "
                  f"{lay['nodes_per_s'] / 1e6:.1f} M nodes/s")
        if args.json:
            import json

            print(json.dumps({"model": args.model, "dataset": args.dataset, **timing}))
    if ref is None:
        print(f"  out shape: {actual.shape} (not checked)")
        return 0
    max_abs = float(np.abs(actual - ref).max())
    print(f"  out shape: {actual.shape}, max abs diff vs torch: {max_abs:.3e}")
    bf16 = lowered.program.feature_dtype == torch.bfloat16
    rtol, atol = (2e-2, 2e-2) if bf16 else (1e-3, 1e-4)
    try:
        np.testing.assert_allclose(actual, ref, rtol=rtol, atol=atol)
    except AssertionError as exc:
        print("FAIL")
        print(exc)
        return 1
    print("PASS")
    return 0


if __name__ == "__main__":
    sys.exit(main())
