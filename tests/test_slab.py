"""Z-slab partition and halo exchange (mogecpp_b200/slab.py), on the CPU.

The partition is checked against the neighbour map: every owned voxel and
every voxel of the inner halo plane has all its neighbours among the rank's
local rows.  The exchange runs as world-size-2 gloo ranks, each running the
oracle's residual block over its local rows between exchanges; the owned
rows must equal the single-process oracle stack bit for bit (each output
row depends only on its neighbours' values, in a fixed order)."""
import os
import time
import socket

import numpy as np
import pytest

from mogecpp_b200 import slab, synth


def _coords(two_samples=False):
    a = synth.small_coords(300, extent=20, grid=48, dilation="z1")
    if not two_samples:
        return a
    b = synth.small_coords(301, extent=16, grid=48, dilation="z1", b=1)
    return synth.dedup_sorted(np.concatenate([a, b]))


def _neighbours(coords):
    from gpu_util import numpy_neighbor_map
    return numpy_neighbor_map(coords)


@pytest.mark.parametrize("nranks", [1, 2, 3, 4])
@pytest.mark.parametrize("two_samples", [False, True])
def test_partition_covers_every_neighbourhood(nranks, two_samples):
    coords = _coords(two_samples)
    n = coords.shape[0]
    parts = slab.partition(coords, nranks)
    assert parts[0].lo == 0 and parts[-1].hi == n
    for p, q in zip(parts[:-1], parts[1:]):
        assert p.hi == q.lo
    nbr = _neighbours(coords)
    sizes = [p.n_owned for p in parts]
    assert max(sizes) < 2.5 * n / nranks  # quantile cuts on plane boundaries
    for p in parts:
        local = set(p.local_rows().tolist())
        assert len(local) == p.n_local
        owned = np.arange(p.lo, p.hi)
        inner = []
        for rows, below in ((p.halo_lo, True), (p.halo_hi, False)):
            if len(rows):
                zs = coords[rows, 2]
                inner.extend(rows[zs == (zs.max() if below else zs.min())].tolist())
        for r in np.concatenate([owned, np.array(inner, dtype=np.int64)]):
            for j in nbr[r]:
                if j < n:
                    assert j in local, (p.rank, r, j)
        # halos hold only other ranks' rows within two planes of the slab
        for rows in (p.halo_lo, p.halo_hi):
            assert np.all((rows < p.lo) | (rows >= p.hi))


def test_partition_send_counts_match_neighbour_halos():
    coords = _coords()
    parts = slab.partition(coords, 3)
    for a, b in zip(parts[:-1], parts[1:]):
        assert a.send_hi == len(b.halo_lo) and b.send_lo == len(a.halo_hi)
        np.testing.assert_array_equal(b.halo_lo, np.arange(a.hi - a.send_hi, a.hi))
        np.testing.assert_array_equal(a.halo_hi, np.arange(b.lo, b.lo + b.send_lo))


def test_partition_rejects_unsorted_or_too_many_ranks():
    coords = _coords()
    with pytest.raises(ValueError):
        slab.partition(coords[::-1].copy(), 2)
    with pytest.raises(ValueError):
        slab.partition(coords, 1000)


def _raw_block(seed, c):
    rng = np.random.default_rng(seed)
    return dict(norm_w=(1 + 0.1 * rng.standard_normal(c)).astype(np.float32),
                norm_b=(0.1 * rng.standard_normal(c)).astype(np.float32),
                w1=synth.conv_weight(seed + 1, c, c), b1=(0.05 * rng.standard_normal(c)).astype(np.float32),
                w2=synth.conv_weight(seed + 2, c, c), b2=(0.05 * rng.standard_normal(c)).astype(np.float32))


def _rank_main(rank, world, port, out_path):
    import torch
    import torch.distributed as dist
    from oracle.oracle import Oracle, W_Q8_0
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        O = Oracle()
        coords = _coords(two_samples=True)
        x = synth.features(310, coords.shape[0], 64)
        part = slab.partition(coords, world)[rank]
        rows = part.local_rows()
        nbr_local = O.make_level(coords[rows])
        xl = torch.from_numpy(x[rows].copy())
        ex = slab.SlabExchange(part, world)
        for blk in range(2):
            ex.exchange(xl)
            xl = torch.from_numpy(O.res_block(xl.numpy(), nbr_local, _raw_block(320 + blk, 64), W_Q8_0))
        np.save(out_path, xl.numpy()[:part.n_owned])
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_match_the_single_process_stack(tmp_path, oracle, world):
    """The owned rows of 2 or 4 gloo ranks (4: two inner ranks with halos on
    both sides, cuts from the balanced partition) equal the single-process
    oracle stack bit for bit."""
    import multiprocessing as mp
    from oracle.oracle import W_Q8_0
    port = _free_port()
    ctx = mp.get_context("spawn")
    outs = [str(tmp_path / f"rank{r}.npy") for r in range(world)]
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, outs[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    coords = _coords(two_samples=True)
    x = synth.features(310, coords.shape[0], 64)
    nbr = oracle.make_level(coords)
    for blk in range(2):
        x = oracle.res_block(x, nbr, _raw_block(320 + blk, 64), W_Q8_0)
    got = np.concatenate([np.load(o) for o in outs])
    np.testing.assert_array_equal(got, x)


def _rank_absent_peer(rank, world, port, out_path):
    """Rank 1 leaves between steps without taking part in the halo exchange;
    rank 0's exchange must end with an error after the process group's short
    timeout instead of waiting for good."""
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    coords = _coords()
    part = slab.partition(coords, world)[rank]
    x = torch.zeros((part.n_local, 8), dtype=torch.float32)
    if rank == 1:
        with open(out_path, "w") as f:
            f.write("left")
        os._exit(0)  # gone before the exchange: no collective in flight
    t0 = time.time()
    try:
        slab.SlabExchange(part, world).exchange(x)
        outcome = "returned"
    except Exception as e:  # noqa: BLE001 - the timeout is the expected outcome
        outcome = "raised:" + type(e).__name__
    with open(out_path, "w") as f:
        f.write(f"{outcome} {time.time() - t0:.1f}")
    os._exit(0)


def test_absent_halo_peer_is_detected_on_the_host(tmp_path):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    outs = [str(tmp_path / f"r{r}.txt") for r in range(2)]
    procs = [ctx.Process(target=_rank_absent_peer, args=(r, 2, port, outs[r])) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert open(outs[1]).read() == "left"
    outcome, secs = open(outs[0]).read().split()
    assert outcome.startswith("raised"), outcome
    assert float(secs) < 60


@pytest.mark.parametrize("nranks", [4, 8])
def test_partition_balances_owned_plus_local_rows(nranks):
    """The cuts even out each rank's work, owned + local rows (conv2 runs over
    the owned rows, conv1 over owned and halo rows), on the 3.1M-voxel shell:
    the busiest rank within 3 % of the mean, where voxel-count quantiles left
    large-plane cuts with large halos."""
    coords = synth.shell_4m_coords()
    parts = slab.partition(coords, nranks)
    work = np.array([p.n_owned + p.n_local for p in parts], dtype=np.float64)
    assert work.max() / work.mean() < 1.03, work
    assert sum(p.n_owned for p in parts) == coords.shape[0]
