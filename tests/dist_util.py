"""Helper: run a function on N local processes with a torch.distributed group
(gloo on CPU; 127.0.0.1 rendezvous) and collect each rank's return value."""
import os
import pickle
import socket
import tempfile
import traceback

import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fn, args, outdir, backend):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), LOCAL_WORLD_SIZE=str(world))
    res = None
    try:
        dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        res = ("ok", fn(rank, world, *args))
    except BaseException as e:  # noqa: BLE001
        res = ("err", f"{type(e).__name__}: {e}\n{traceback.format_exc()}")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass
    with open(os.path.join(outdir, f"{rank}.pkl"), "wb") as f:
        pickle.dump(res, f)


def run_dist(fn, world=2, args=(), backend="gloo", timeout=120):
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_worker, args=(r, world, port, fn, args, d, backend)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout)
            if p.is_alive():
                p.kill()
        out = []
        for r in range(world):
            path = os.path.join(d, f"{r}.pkl")
            if not os.path.exists(path):
                raise RuntimeError(f"rank {r} produced no result")
            with open(path, "rb") as f:
                status, val = pickle.load(f)
            if status != "ok":
                raise RuntimeError(f"rank {r} failed: {val}")
            out.append(val)
        return out
