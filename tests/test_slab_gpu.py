"""Z-slab residual stack on two GPUs: one process per GPU, NCCL halo
exchange before each Q8_0 residual block (mogecpp_b200/slab.py); for the
GroupNorm block the sample-wide statistics are also all-reduced over NCCL.  The owned
rows of the two ranks are compared with the single-GPU stack over the whole
set and with the oracle.  The conv sums each row's taps in one fixed order
whatever its tile, so the LayerNorm stack's owned rows equal the single-GPU
rows bit for bit; the GroupNorm block's sample statistics are double sums
in another order (rel-L2 ~1e-6 after the float conversion).  A wrong halo
would put O(1) errors on the rows next to the slab boundary.  Skipped with
fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

from mogecpp_b200 import slab, synth

pytestmark = pytest.mark.gpu


def _coords():
    return synth.small_coords(330, extent=40, grid=64, dilation="z1")


def _raw_block(seed, c):
    rng = np.random.default_rng(seed)
    r = dict(norm_w=(1 + 0.1 * rng.standard_normal(c)).astype(np.float32),
             norm_b=(0.1 * rng.standard_normal(c)).astype(np.float32),
             w1=synth.conv_weight(seed + 1, c, c), b1=(0.05 * rng.standard_normal(c)).astype(np.float32),
             w2=synth.conv_weight(seed + 2, c, c), b2=(0.05 * rng.standard_normal(c)).astype(np.float32))
    r["gn_w"], r["gn_b"] = r["norm_w"], r["norm_b"]
    return r


def _stack(ex, coords_np, x_np, block, world=1, part=None, exchange=None, plan_kind=None):
    import torch
    from mogecpp_b200.synth import quantize_q8_0
    dev = torch.device("cuda", torch.cuda.current_device())
    cd = torch.from_numpy(coords_np).to(dev)
    nbr = ex.make_level(cd)
    plan = ex.conv_plan(cd, nbr, plan_kind) if plan_kind else None
    x = torch.from_numpy(x_np).to(dev)
    for blk in range(2):
        raw = _raw_block(340 + blk, 128)
        b = dict(norm_w=torch.from_numpy(raw["norm_w"]).to(dev), norm_b=torch.from_numpy(raw["norm_b"]).to(dev),
                 gn_w=torch.from_numpy(raw["gn_w"]).to(dev), gn_b=torch.from_numpy(raw["gn_b"]).to(dev),
                 b1=torch.from_numpy(raw["b1"]).to(dev), b2=torch.from_numpy(raw["b2"]).to(dev),
                 w1=ex.prepare_weight(torch.from_numpy(quantize_q8_0(raw["w1"])).to(dev), "q8_0", 128, 128, 27),
                 w2=ex.prepare_weight(torch.from_numpy(quantize_q8_0(raw["w2"])).to(dev), "q8_0", 128, 128, 27))
        if exchange is not None:
            exchange.exchange(x)
        if block == "gn":
            import torch.distributed as dist
            ex.res_block_gn(x, nbr, cd, 1, b, plan=plan, n_stat=part.n_owned if part else None,
                            allreduce=(lambda t: dist.all_reduce(t)) if world > 1 else None)
        else:
            ex.res_block(x, nbr, b, plan=plan)
    ex.check()
    return x.float().cpu().numpy()


def _rank_main(rank, world, port, out_path, block):
    import torch
    import torch.distributed as dist
    from mogecpp_b200.sparse import SparseCudaExecutor
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        ex = SparseCudaExecutor(rank)
        coords = _coords()
        part = slab.partition(coords, world)[rank]
        rows = part.local_rows()
        x = synth.features_rows(331, rows, 128, np.float16)
        y = _stack(ex, np.ascontiguousarray(coords[rows]), x, block, world, part, slab.SlabExchange(part, world),
                   plan_kind="tap_order")
        np.save(out_path, y[:part.n_owned])
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("block", ["ln", "gn"])
def test_two_gpu_slabs_match_single_gpu_stack(tmp_path, ex, oracle, block):
    import multiprocessing as mp
    import torch
    from conftest import max_abs, rel_l2
    from oracle.oracle import W_Q8_0
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    outs = [str(tmp_path / f"rank{r}.npy") for r in range(world)]
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, outs[r], block)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = np.concatenate([np.load(o) for o in outs])
    coords = _coords()
    x = synth.features(331, coords.shape[0], 128, np.float16)
    single = _stack(ex, coords, x, block)
    if block == "ln":
        # every row's taps are summed in one order in any tile: the owned rows
        # of the slabs are the single-GPU rows bit for bit
        np.testing.assert_array_equal(got, single)
    # GroupNorm: the statistics are double sums in another order (per-rank
    # partial sums, then the all-reduce)
    assert rel_l2(got, single) < 1e-3 and max_abs(got, single) < 3e-2, (rel_l2(got, single), max_abs(got, single))
    # rows of the two planes on either side of the cut
    cut = slab.partition(coords, world)[1].lo
    zc = coords[cut, 2]
    near = np.flatnonzero(np.abs(coords[:, 2] - zc) <= 2)
    assert max_abs(got[near], single[near]) < 3e-2
    nbr = oracle.make_level(coords)
    h = x.astype(np.float32)
    for blk in range(2):
        raw = _raw_block(340 + blk, 128)
        h = (oracle.res_block_gn(h, nbr, coords[:, 3], raw, W_Q8_0) if block == "gn"
             else oracle.res_block(h, nbr, raw, W_Q8_0))
        h = h.astype(np.float16).astype(np.float32)
    assert rel_l2(got, h) < 3e-3 and max_abs(got, h) < 3e-2


def _rank_main_peer(rank, world, port, out_path):
    import torch
    import torch.distributed as dist
    from mogecpp_b200.sparse import SparseCudaExecutor
    from mogecpp_b200.synth import quantize_q8_0
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    ps = None
    try:
        ex = SparseCudaExecutor(rank)
        coords = _coords()
        part = slab.partition(coords, world)[rank]
        rows = part.local_rows()
        dev = torch.device("cuda", rank)
        cd = torch.from_numpy(np.ascontiguousarray(coords[rows])).to(dev)
        x = torch.from_numpy(synth.features_rows(331, rows, 128, np.float16)).to(dev)
        ps = slab.PeerSlab(ex, part, world)
        ps.set_level(cd)
        ps.put_features(x)
        for blk in range(2):
            raw = _raw_block(340 + blk, 128)
            b = dict(norm_w=torch.from_numpy(raw["norm_w"]).to(dev), norm_b=torch.from_numpy(raw["norm_b"]).to(dev),
                     b1=torch.from_numpy(raw["b1"]).to(dev), b2=torch.from_numpy(raw["b2"]).to(dev),
                     w1=ex.prepare_weight(torch.from_numpy(quantize_q8_0(raw["w1"])).to(dev), "q8_0", 128, 128, 27),
                     w2=ex.prepare_weight(torch.from_numpy(quantize_q8_0(raw["w2"])).to(dev), "q8_0", 128, 128, 27))
            ps.res_block(b)
        out = torch.empty((part.n_owned, 128), dtype=torch.float16, device=dev)
        ps.get_features(out)
        ex.check()
        np.save(out_path, out.float().cpu().numpy())
        dist.barrier()
    finally:
        if ps is not None:
            ps.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_peer_halo_matches_single_gpu_stack(tmp_path, ex, world):
    """The fused-exchange path (msc_slab_*): halo rows written by each
    block's second conv into the neighbours' buffers over NVLink.  The owned
    rows of every rank equal the single-GPU stack bit for bit.  With four
    ranks the two inner ones exchange with both neighbours."""
    import multiprocessing as mp
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    outs = [str(tmp_path / f"peer{r}.npy") for r in range(world)]
    procs = [ctx.Process(target=_rank_main_peer, args=(r, world, port, outs[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = np.concatenate([np.load(o) for o in outs])
    coords = _coords()
    single = _stack(ex, coords, synth.features(331, coords.shape[0], 128, np.float16), "ln", plan_kind="tap_order")
    np.testing.assert_array_equal(got, single)
