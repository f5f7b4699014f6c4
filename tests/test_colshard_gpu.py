"""Column-sharded prefill on two GPUs: the all-gather fused into the GEMM / SiLU*mul kernels (peer
stores over NVLink) and the NCCL all-gather variant.

* fused and NCCL run the same kernels with the same launch shapes on the same inputs: their outputs
  must be bit-identical, on both ranks;
* end to end against the unsharded stack on one GPU within the north-star tolerance (max relative
  error 2e-3, per-row cosine 0.99999) over two layers. The sharded GEMMs split K differently from
  the unsharded ones, so fp16 outputs differ in the last bit, and the synthetic stack amplifies
  such differences with depth (already ~9e-3 at four layers between fp32 and fp64 accumulation on
  the CPU), so depth beyond two layers is checked projection by projection instead:
* the last layer's gathered buffers (every rank's column slice in place) against one-GPU matmuls of
  the same gathered inputs, within the tolerance;
* the fused forward captured in a CUDA graph (the barrier counts its epochs on the device) and
  replayed twice gives the eager result bit for bit.
Skipped when fewer than two GPUs are visible."""
import importlib
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

N_LAYERS, M = 2, 256


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    import datetime
    import sys

    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "tests"))
    sys.path.insert(0, root)
    from conftest import load_package

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        pkg = load_package()
        serve = importlib.import_module("strands_decider_web_b200.serve")
        ctx = pkg.Context(rank)
        x = torch.from_numpy(np.random.default_rng(11).standard_normal((M, serve.HIDDEN)).astype(np.float16)).cuda()
        fused = serve.FusedColshardStack(ctx, None, rank, world, max_tokens=M, n_layers=N_LAYERS)
        y_fused = fused.forward(x).clone()
        torch.cuda.synchronize()
        y_graph = fused.capture(x)  # the same forward recorded as one CUDA graph, barriers included
        fused.replay()
        fused.replay()
        torch.cuda.synchronize()
        y_graph = y_graph.cpu().numpy()
        gathered = {k: fused._view(k, M, w).clone() for k, w in fused.widths.items()}
        sharded = serve.CudaStack(ctx, N_LAYERS, rank, world)
        y_nccl = sharded.forward(x)
        torch.cuda.synchronize()
        errs = ctx.check_errors()
        out = {"fused": y_fused.cpu().numpy(), "nccl": y_nccl.cpu().numpy(), "graph": y_graph, "errs": errs}
        if rank == 0:
            full = serve.CudaStack(ctx, N_LAYERS)
            out["ref"] = full.forward(x).cpu().numpy()
            last = full.layers[-1]
            out["b"] = (gathered["b"].cpu().numpy(),
                        ctx.matmul(gathered["a"][:, :serve.HIDDEN].contiguous(), last["out_proj"]).cpu().numpy())
            out["d"] = (gathered["d"].cpu().numpy(), ctx.matmul(gathered["mid"], last["down"]).cpu().numpy())
        fused.close()
        q.put((rank, out))
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_fused_and_nccl_colshard_match_single_gpu(world):
    """Two and four ranks (narrower slices per rank: 24 gate|up n-blocks at four)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import s4ref
    mp = torch.multiprocessing.get_context("spawn")
    q = mp.Queue()
    port = _free_port()
    procs = [mp.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ref = res[0]["ref"].astype(np.float32)
    for r in range(world):
        assert res[r]["errs"] == 0
        np.testing.assert_array_equal(res[r]["fused"], res[r]["nccl"])
        np.testing.assert_array_equal(res[r]["fused"], res[r]["graph"])
        ok, mr, mc = s4ref.check(res[r]["fused"], ref)
        assert ok, (r, mr, mc)
    for r in range(1, world):
        np.testing.assert_array_equal(res[0]["fused"], res[r]["fused"])
    for key in ("b", "d"):
        got, want = res[0][key]
        ok, mr, mc = s4ref.check(got, want.astype(np.float32))
        assert ok, (key, mr, mc)
