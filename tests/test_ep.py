"""Expert parallelism (laii_b200.ep).

CPU: shard bookkeeping, and the whole exchange logic with two gloo ranks and
the oracle as the expert compute (bit-exact against the single-process oracle
layer).  GPU: the lfm_gpu_moe_ep_* path through the C-ABI, against the regular
forward -- on one GPU as a world of one, and as a world of two (two handles,
one per "rank", exchanging through an in-process mailbox; these kernels never
wait on one another, so sharing one GPU is safe).
"""
import os
import socket
import threading

import numpy as np
import pytest
import torch

from conftest import cached_layer, rel_l2
from laii_b200 import ep

REL_L2, MAX_ABS = 1e-3, 5e-3


class OracleOps:
    """Test-only ops: the CPU oracle restatement as route / experts / combine."""

    def __init__(self, L, first, count):
        from oracle.oracle import Oracle
        self.o = Oracle()
        self.L, self.first, self.count = L, first, count

    def route(self, layer, x):
        idx, w, q8 = self.o.ep_route(self.L, x.numpy())
        return torch.from_numpy(idx), torch.from_numpy(w), torch.from_numpy(q8)

    def experts(self, layer, q8, ids):
        return torch.from_numpy(self.o.ep_expert_rows(self.L, self.first, self.count, q8.numpy(), ids.numpy()))

    def combine(self, layer, x, w, y):
        self.o.ep_combine(x.numpy(), w.numpy(), y.numpy())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shards_tile_the_experts():
    for E in (1, 7, 32, 64, 256):
        for world in (1, 2, 3, 8):
            if world > E:
                continue
            seen = []
            sizes = []
            for r in range(world):
                first, n = ep.shard_of(E, world, r)
                seen += list(range(first, first + n))
                sizes.append(n)
            assert seen == list(range(E))
            assert max(sizes) - min(sizes) <= 1
            owners = ep.owner_of(torch.arange(E), E, world).tolist()
            for r in range(world):
                first, n = ep.shard_of(E, world, r)
                assert owners[first:first + n] == [r] * n


D, E, K, I, T_PER_RANK = 512, 8, 2, 512, 5


def _gloo_rank(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    from laii_b200 import synth
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        L = synth.make_moe_layer(D, E, K, I, layer=3)
        x_all = synth.make_hidden(world * T_PER_RANK, D, seed_offset=5)
        x = torch.from_numpy(np.array(x_all[rank * T_PER_RANK:(rank + 1) * T_PER_RANK], copy=True))
        first, count = ep.shard_of(E, world, rank)
        ep.ep_forward(OracleOps(L, first, count), ep.TorchComm(), 0, x, E, K)
        np.save(os.path.join(out_dir, f"x{rank}.npy"), x.numpy())
    finally:
        dist.destroy_process_group()


def test_ep_two_gloo_ranks_equal_the_single_rank_oracle(tmp_path):
    import torch.multiprocessing as mp
    from laii_b200 import synth
    from oracle.oracle import Oracle
    world = 2
    mp.spawn(_gloo_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    got = np.concatenate([np.load(tmp_path / f"x{r}.npy") for r in range(world)])
    L = synth.make_moe_layer(D, E, K, I, layer=3)
    want, _, _, _, _ = Oracle().moe_forward(L, synth.make_hidden(world * T_PER_RANK, D, seed_offset=5))
    assert np.array_equal(got, want)


class MailboxComm:
    """A world of `world` ranks as threads of one process (GPU tensors handed over in memory)."""

    def __init__(self, world, rank, box, barrier):
        self.world, self.rank, self.box, self.barrier = world, rank, box, barrier

    def exchange(self, send, send_counts, recv_counts=None):
        torch.cuda.synchronize()
        offs = np.cumsum([0] + list(send_counts))
        for dst in range(self.world):
            self.box[(self.rank, dst)] = send[offs[dst]:offs[dst + 1]]
        self.barrier.wait()
        parts = [self.box[(src, self.rank)] for src in range(self.world)]
        self.barrier.wait()
        return torch.cat(parts), [p.shape[0] for p in parts]


@pytest.mark.gpu
@pytest.mark.parametrize("world,T", [(1, 8), (2, 6), (4, 3)])
def test_ep_on_one_gpu_matches_forward(world, T):
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE
    Dg, Eg, Kg, Ig = 2048, 32, 4, 1792
    L = cached_layer(Dg, Eg, Kg, Ig)
    x_all = synth.make_hidden(world * T, Dg, seed_offset=31)
    ref_h = GpuMoE(0)
    ref_h.upload_layer(0, L)
    want = ref_h.forward(0, np.array(x_all, copy=True))
    ref_h.close()
    handles = []
    for r in range(world):
        g = GpuMoE(0)
        first, count = ep.shard_of(Eg, world, r)
        g.upload_layer_shard(0, L, first, count)
        handles.append(g)
    box, barrier = {}, threading.Barrier(world)
    outs = [None] * world
    errs = []

    def run(r):
        try:
            torch.cuda.set_device(0)
            x = torch.from_numpy(np.array(x_all[r * T:(r + 1) * T], copy=True)).cuda()
            comm = ep.LocalComm() if world == 1 else MailboxComm(world, r, box, barrier)
            ep.ep_forward(ep.GpuOps(handles[r], Dg, Kg), comm, 0, x, Eg, Kg)
            torch.cuda.synchronize()
            handles[r].sync()
            outs[r] = x.cpu().numpy()
        except Exception as e:  # surfaced below
            errs.append(e)
            barrier.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    for g in handles:
        g.close()
    assert not errs, errs
    got = np.concatenate(outs)
    assert rel_l2(got, want) <= REL_L2
    assert float(np.abs(got - want).max()) <= MAX_ABS


@pytest.mark.gpu
def test_shard_layer_refuses_the_regular_forward():
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE, MoEError
    L = cached_layer(2048, 32, 4, 1792)
    with GpuMoE(0) as g:
        g.upload_layer_shard(0, L, 8, 8)
        with pytest.raises(MoEError) as ei:
            g.forward(0, synth.make_hidden(2, 2048))
        assert ei.value.status == -2


@pytest.mark.gpu
def test_synth_shard_matches_the_full_layer_bytes():
    from laii_b200.moe import GpuMoE
    import bench
    D_, E_, K_, I_ = 2048, 32, 4, 1792
    per_gu = I_ * (D_ // 256) * 144
    with GpuMoE(0) as g:
        g.synth_layer(0, D_, E_, K_, I_, bench.layer_seeds(0))
        g.synth_layer_shard(1, D_, E_, K_, I_, bench.layer_seeds(0), 20, 4)
        full = g.read_layer(0, "gate", E_ * per_gu)
        part = g.read_layer(1, "gate", 4 * per_gu)
        assert np.array_equal(full[20 * per_gu:24 * per_gu], part)


def _nccl_rank(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        Dg, Eg, Kg, Ig, T = 2048, 32, 4, 1792, 24
        L = synth.make_moe_layer(Dg, Eg, Kg, Ig, layer=7)
        x_all = synth.make_hidden(world * T, Dg, seed_offset=61)
        g = GpuMoE(rank)
        first, count = ep.shard_of(Eg, world, rank)
        g.upload_layer_shard(0, L, first, count)
        x = torch.from_numpy(np.array(x_all[rank * T:(rank + 1) * T], copy=True)).cuda()
        ep.ep_forward(ep.GpuOps(g, Dg, Kg), ep.TorchComm(), 0, x, Eg, Kg)
        torch.cuda.synchronize()
        g.sync()
        np.save(os.path.join(out_dir, f"x{rank}.npy"), x.cpu().numpy())
        g.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_ep_nccl_two_gpus_match_single_gpu_forward(tmp_path):
    """Expert parallelism across two GPUs (NCCL all-to-all) against the one-GPU layer."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE
    world, T = 2, 24
    mp.spawn(_nccl_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    got = np.concatenate([np.load(tmp_path / f"x{r}.npy") for r in range(world)])
    L = synth.make_moe_layer(2048, 32, 4, 1792, layer=7)
    with GpuMoE(0) as g:
        g.upload_layer(0, L)
        want = g.forward(0, synth.make_hidden(world * T, 2048, seed_offset=61))
    assert rel_l2(got, want) <= REL_L2
    assert float(np.abs(got - want).max()) <= MAX_ABS


# ---- expert parallelism over peer memory (lfm_gpu_moe_ep_p2p_*) ----------

P2P_SHAPE = (2048, 32, 4, 1792)


def _p2p_layers(g, n_layers, first, count, shape=P2P_SHAPE):
    import bench
    D_, E_, K_, I_ = shape
    for l in range(n_layers):
        if count == E_:
            g.synth_layer_shard(l, D_, E_, K_, I_, bench.layer_seeds(l + 40), 0, E_)
        else:
            g.synth_layer_shard(l, D_, E_, K_, I_, bench.layer_seeds(l + 40), first, count)


def _p2p_want(xs, n_layers, shape=P2P_SHAPE):
    """Every step of the test through the one-GPU forward of the full layers."""
    import bench
    from laii_b200.moe import GpuMoE
    D_, E_, K_, I_ = shape
    out = []
    with GpuMoE(0) as g:
        for l in range(n_layers):
            g.synth_layer(l, D_, E_, K_, I_, bench.layer_seeds(l + 40))
        for x in xs:
            y = np.array(x, copy=True)
            for l in range(n_layers):
                if y.shape[0]:
                    y = g.forward(l, y)
            out.append(y)
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("Ts", [(8, 24, 0, 300), (64, 1), (1100, 40)])
def test_ep_p2p_world_of_one_matches_forward(Ts):
    """The peer-memory layer step as a world of one (every exchange to itself), two layers a step,
    against the regular forward: the same grouped GEMMs and k-ordered combine, so bit-exact."""
    import torch
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE
    D_, E_, K_, I_ = P2P_SHAPE
    xs = [synth.make_hidden(T, D_, seed_offset=77 + T) if T else np.zeros((0, D_), np.float32) for T in Ts]
    want = _p2p_want(xs, 2)
    with GpuMoE(0) as g:
        _p2p_layers(g, 2, 0, E_)
        assert ep.p2p_connect(g, max(Ts), D_, E_, K_, I_) == (0, 1)
        for x, wnt in zip(xs, want):
            xd = torch.from_numpy(np.array(x, copy=True)).cuda()
            s = torch.cuda.current_stream().cuda_stream
            for l in range(2):
                g.ep_p2p_forward(l, xd.data_ptr() if xd.numel() else 0, xd.shape[0], s)
            torch.cuda.synchronize()
            g.sync()
            got = xd.cpu().numpy()
            assert np.array_equal(got, wnt)
        g.ep_p2p_detach()


@pytest.mark.gpu
def test_ep_p2p_bounded_wait_reports_timeout_and_recovers():
    """A wait on a step no rank signals runs out after wait_ms: TIMEOUT at the next sync, the context
    stays usable and the next layer step is still right."""
    import time
    import torch
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE, MoEError
    D_, E_, K_, I_ = P2P_SHAPE
    x = synth.make_hidden(24, D_, seed_offset=5)
    want = _p2p_want([x], 1)[0]
    with GpuMoE(0) as g:
        _p2p_layers(g, 1, 0, E_)
        ep.p2p_connect(g, 24, D_, E_, K_, I_, wait_ms=200)
        g.ep_p2p_wait_check(torch.cuda.current_stream().cuda_stream)
        t0 = time.perf_counter()
        with pytest.raises(MoEError) as ei:
            g.sync()
        assert ei.value.status == -9
        assert time.perf_counter() - t0 < 10.0
        xd = torch.from_numpy(np.array(x, copy=True)).cuda()
        g.ep_p2p_forward(0, xd.data_ptr(), 24, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        g.sync()
        assert np.array_equal(xd.cpu().numpy(), want)


P2P_STEPS = [(40, 7), (0, 33), (200, 200)]  # tokens of rank 0, rank 1 per step


def _p2p_rank(rank, world, port, out_dir, shape):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    try:
        D_, E_, K_, I_ = shape
        first, count = ep.shard_of(E_, world, rank)
        g = GpuMoE(rank)
        _p2p_layers(g, 2, first, count, shape)
        Tmax = max(max(s) for s in P2P_STEPS)
        ep.p2p_connect(g, Tmax, D_, E_, K_, I_, wait_ms=10000)
        for i, Ts in enumerate(P2P_STEPS):
            T = Ts[rank]
            x = synth.make_hidden(T, D_, seed_offset=1000 * i + 100 * rank) if T else np.zeros((0, D_), np.float32)
            xd = torch.from_numpy(np.array(x, copy=True)).cuda()
            s = torch.cuda.current_stream().cuda_stream
            for l in range(2):
                g.ep_p2p_forward(l, xd.data_ptr() if T else 0, T, s)
            torch.cuda.synchronize()
            g.sync()
            np.save(os.path.join(out_dir, f"p2p_{i}_{rank}.npy"), xd.cpu().numpy())
        # the same steps through the stack call: captured on first use, then graph replays
        xbuf = torch.zeros((Tmax, D_), dtype=torch.float32, device="cuda")
        for rep in range(3):
            for i, Ts in enumerate(P2P_STEPS):
                T = Ts[rank]
                if T:
                    xbuf[:T].copy_(torch.from_numpy(synth.make_hidden(T, D_, seed_offset=1000 * i + 100 * rank)))
                g.ep_p2p_forward_stack(0, 2, xbuf.data_ptr() if T else 0, T, torch.cuda.current_stream().cuda_stream)
                torch.cuda.synchronize()
                g.sync()
                np.save(os.path.join(out_dir, f"p2ps_{rep}_{i}_{rank}.npy"), xbuf[:T].cpu().numpy())
        dist.barrier()
        g.ep_p2p_detach()
        g.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [P2P_SHAPE, (2048, 64, 4, 1536)])
def test_ep_p2p_two_gpus_match_single_gpu_forward(tmp_path, shape):
    """Two processes, one GPU each, experts split in half (the config 1-4 and the config 5 layer
    shapes): uneven and empty token counts per rank, two layers a step, three steps; each rank's
    tokens against the one-GPU forward, bit-exact."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from laii_b200 import synth
    world = 2
    mp.spawn(_p2p_rank, args=(world, _free_port(), str(tmp_path), tuple(shape)), nprocs=world, join=True)
    D_ = shape[0]
    for i, Ts in enumerate(P2P_STEPS):
        xs = [synth.make_hidden(T, D_, seed_offset=1000 * i + 100 * r) if T else np.zeros((0, D_), np.float32)
              for r, T in enumerate(Ts)]
        want = _p2p_want(xs, 2, shape)
        for r in range(world):
            got = np.load(tmp_path / f"p2p_{i}_{r}.npy")
            assert np.array_equal(got, want[r]), (i, r)
            for rep in range(3):
                got = np.load(tmp_path / f"p2ps_{rep}_{i}_{r}.npy")
                assert np.array_equal(got, want[r]), ("stack", rep, i, r)


@pytest.mark.gpu
def test_ep_p2p_stack_world_of_one_with_dense_layer_replays():
    """A dense layer and two MoE shard layers through the expert-parallel stack call (world of one):
    first call eager + capture, later calls CUDA-graph replays with the device-side step counter,
    against the regular stack forward."""
    import torch
    import bench
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE
    from conftest import cached_dense
    D_, E_, K_, I_ = P2P_SHAPE
    dense = cached_dense(D_, 7168)
    x = synth.make_hidden(24, D_, seed_offset=9)
    with GpuMoE(0) as ref:
        ref.upload_dense(0, dense)
        for l in (1, 2):
            ref.synth_layer(l, D_, E_, K_, I_, bench.layer_seeds(l + 40))
        want = ref.forward_stack(0, 3, np.array(x, copy=True))
    with GpuMoE(0) as g:
        g.upload_dense(0, dense)
        for l in (1, 2):
            g.synth_layer_shard(l, D_, E_, K_, I_, bench.layer_seeds(l + 40), 0, E_)
        ep.p2p_connect(g, 24, D_, E_, K_, I_)
        xbuf = torch.empty((24, D_), dtype=torch.float32, device="cuda")
        for rep in range(4):
            xbuf.copy_(torch.from_numpy(x))
            g.ep_p2p_forward_stack(0, 3, xbuf.data_ptr(), 24, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            g.sync()
            assert np.array_equal(xbuf.cpu().numpy(), want), rep


@pytest.mark.gpu
def test_ep_p2p_connect_refuses_handles_of_other_shapes():
    """Every rank computes the arena layout from its own attach arguments, so a handle attached with
    other shapes (here max_tokens) is refused before anything is mapped."""
    from laii_b200.moe import GpuMoE, MoEError
    D_, E_, K_, I_ = P2P_SHAPE
    with GpuMoE(0) as a, GpuMoE(0) as b:
        ha = a.ep_p2p_attach(0, 1, 24, D_, E_, K_, I_)
        hb = b.ep_p2p_attach(0, 1, 32, D_, E_, K_, I_)
        assert len(ha) == len(hb) == GpuMoE.IPC_HANDLE_BYTES
        with pytest.raises(MoEError) as ei:
            a.ep_p2p_connect([hb])
        assert ei.value.status == -1 and "max_tokens 32" in str(ei.value)
        a.ep_p2p_connect([ha])  # its own handle still connects
        a.ep_p2p_detach()
        b.ep_p2p_detach()
