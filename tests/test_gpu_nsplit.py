"""GPU, 2 ranks (skipped with fewer GPUs): the N-split with the all-gather fused into the GEMM
epilogue (envg_linear_nsplit).  Each rank holds one output-column shard of W and writes its
columns into both ranks' copies of Y -- by peer stores and, where the NVSwitch offers it, by one
NVLS multimem store -- and every rank then holds the full Y, bit-identical to the unsplit
linear computed on one GPU."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    from datetime import timedelta

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem

    from invision_b200 import envg
    from invision_b200.nsplit import shard_bounds
    from tests.common import inputs

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    results = []
    try:
        envg.init(rank)
        dev = torch.device("cuda", rank)
        for (M, K, N, gate_up) in [(300, 512, 1040, False), (257, 256, 2 * 392, True), (40, 1024, 768, False),
                                   (5, 768, 520, False)]:
            x, w, b = inputs(M, K, N, seed=M + K + N)
            half = N // 2 if gate_up else N
            n0, n1, per = shard_bounds(half, world, rank, 128)
            layout = envg.LAYOUT_GATE_UP if gate_up else envg.LAYOUT_PLAIN
            Ws = envg.Weight(w, layout=layout, shard=(n0, n1))
            bs = np.concatenate([b[n0:n1], b[half + n0:half + n1]]) if gate_up else b[n0:n1]
            xt = torch.from_numpy(x).to(dev)
            bt = torch.from_numpy(np.ascontiguousarray(bs)).to(dev)
            Y = symm_mem.empty(M, half, device=dev)
            hdl = symm_mem.rendezvous(Y, dist.group.WORLD)
            modes = [("p2p", list(hdl.buffer_ptrs), 0)]
            if hdl.has_multicast_support and hdl.multicast_ptr:
                modes.append(("multicast", None, hdl.multicast_ptr))
            Wf = envg.Weight(w, layout=layout)
            ref = torch.empty(M, half, device=dev)
            envg.linear(ref, xt, Wf, bias=torch.from_numpy(b).to(dev))
            torch.cuda.synchronize()
            for name, peers, mc in modes:
                Y.fill_(float("nan"))
                torch.cuda.synchronize()
                hdl.barrier()
                envg.linear_nsplit(Y, xt, Ws, n0, peers=peers, multicast=mc, bias=bt)
                torch.cuda.synchronize()
                hdl.barrier()
                ok = bool(torch.equal(Y, ref))
                results.append((f"{name} {M}x{K}x{N} gate_up={gate_up}", ok))
            if not gate_up and M > 64:
                # gated residual: every copy of Y starts as the same residual h0
                rng = np.random.default_rng(M)
                h0 = torch.from_numpy(rng.standard_normal((M, half)).astype(np.float32)).to(dev)
                gate = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(dev)
                ref_r = h0.clone()
                envg.linear(ref_r, xt, Wf, bias=torch.from_numpy(b).to(dev), epilogue=envg.EPI_GATED_RESIDUAL,
                            gate=gate)
                gs = gate[n0:n1].contiguous()
                for name, peers, mc in modes:
                    Y.copy_(h0)
                    torch.cuda.synchronize()
                    hdl.barrier()
                    envg.linear_nsplit(Y, xt, Ws, n0, peers=peers, multicast=mc, bias=bt,
                                       epilogue=envg.EPI_GATED_RESIDUAL, gate=gs)
                    torch.cuda.synchronize()
                    hdl.barrier()
                    results.append((f"{name} gated residual {M}x{K}x{N}", bool(torch.equal(Y, ref_r))))
            Ws.free()
            Wf.free()
            del Y, hdl
        # envg_linear_nsplit_batch: two shards (plain + SiLU-gate) in one call, bit-identical
        # to one GPU; the second reads the same input, so it is cast once
        M, K = 384, 512
        x, w1, b1 = inputs(M, K, 640, seed=11)
        _, w2, b2 = inputs(M, K, 2 * 512, seed=12)
        xt = torch.from_numpy(x).to(dev)
        calls, refs, keep = [], [], []
        for w, b, gate_up in ((w1, b1, False), (w2, b2, True)):
            N = w.shape[0]
            half = N // 2 if gate_up else N
            n0, n1, per = shard_bounds(half, world, rank, 128)
            layout = envg.LAYOUT_GATE_UP if gate_up else envg.LAYOUT_PLAIN
            Ws = envg.Weight(w, layout=layout, shard=(n0, n1))
            bs = np.concatenate([b[n0:n1], b[half + n0:half + n1]]) if gate_up else b[n0:n1]
            Y = symm_mem.empty(M, half, device=dev)
            hdl = symm_mem.rendezvous(Y, dist.group.WORLD)
            Wf = envg.Weight(w, layout=layout)
            ref = torch.empty(M, half, device=dev)
            envg.linear(ref, xt, Wf, bias=torch.from_numpy(b).to(dev))
            Wf.free()
            Y.fill_(float("nan"))
            calls.append(dict(y=Y, x=xt, W=Ws, col0=n0, peers=list(hdl.buffer_ptrs),
                              bias=torch.from_numpy(np.ascontiguousarray(bs)).to(dev)))
            refs.append(ref)
            keep.append((Ws, hdl))
        # a third shard kept on its rank (no peers: ENVG_KEEP_SHARDED semantics), head-aligned
        from invision_b200.nsplit import segment_rows

        _, w3, _ = inputs(M, K, 4 * 256, seed=13)
        rows = segment_rows((256, 256, 256, 256), world, rank, 128)
        W3 = envg.Weight(np.ascontiguousarray(w3[rows]))
        Wf3 = envg.Weight(w3)
        ref3 = torch.empty(M, 4 * 256, device=dev)
        envg.linear(ref3, xt, Wf3)
        Wf3.free()
        y3 = torch.full((M, len(rows)), float("nan"), device=dev)
        calls.append(dict(y=y3, x=xt, W=W3, col0=0))
        refs.append(ref3[:, torch.from_numpy(rows).to(dev)])
        keep.append((W3, None))
        torch.cuda.synchronize()
        keep[1][1].barrier()
        envg.linear_nsplit_batch(calls)
        torch.cuda.synchronize()
        keep[1][1].barrier()
        for i, (c, ref) in enumerate(zip(calls, refs)):
            results.append((f"nsplit batch item {i}", bool(torch.equal(c["y"], ref))))
        for Ws, _ in keep:
            Ws.free()
        del calls, keep
        if rank == 0:
            q.put(results)
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_nsplit_fused_gather_two_ranks():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    res = q.get(timeout=5)
    bad = [name for name, ok in res if not ok]
    assert not bad and len(res) >= 4, res


@pytest.mark.parametrize("M", [2048, 300, 16, 4])
def test_kept_shard_writes_only_its_columns(gpu, M):
    """ENVG_KEEP_SHARDED on one GPU: the shard's columns land in [col0, col0 + width) of the
    rank's own Y (every GEMM path: CTA-pair, k2_set, k_gemv), bit-identical to the same columns of
    the unsplit linear, and nothing else of Y is written."""
    import torch

    from tests.common import inputs

    envg = gpu
    K, N = 512, 1024
    x, w, b = inputs(M, K, N, seed=M + 3)
    n0, n1 = 256, 640
    Ws = envg.Weight(w, shard=(n0, n1))
    Wf = envg.Weight(w)
    xt = torch.from_numpy(x).cuda()
    bt = torch.from_numpy(b).cuda()
    ref = torch.empty(M, N, device="cuda")
    envg.linear(ref, xt, Wf, bias=bt)
    for how in ("flag", "no peers"):
        Y = torch.full((M, N), 7.0, device="cuda")
        if how == "flag":
            L = envg.lib()
            rc = L.envg_linear_nsplit(Y.data_ptr(), None, 0, None, N, n0, xt.data_ptr(), Ws.h,
                                      bt[n0:n1].contiguous().data_ptr(), M, K, n1 - n0, envg.EPI_BIAS, None,
                                      envg.DEVICE_PTRS | envg.KEEP_SHARDED)
            assert rc == envg.OK, envg.last_error()
        else:
            envg.linear_nsplit_batch([dict(y=Y, x=xt, W=Ws, col0=n0, bias=bt[n0:n1].contiguous())])
        torch.cuda.synchronize()
        assert torch.equal(Y[:, n0:n1], ref[:, n0:n1]), how
        assert bool((Y[:, :n0] == 7.0).all()) and bool((Y[:, n1:] == 7.0).all()), how
    Ws.free()
    Wf.free()
