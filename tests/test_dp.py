"""Data-parallel training step: ranks each take a slice of the batch, per-block gradient buckets are summed across
ranks during the backward (checkpointed blocks) and the tail bucket after it, and AdamW divides by the world size.
With equal token counts per rank this equals one full-batch step (Training.cs:81-104 semantics on the union batch).

CPU tests run 2 gloo ranks over the oracle (the trainer's bucket logic with a host all-reduce); the GPU test runs
2 NCCL ranks over the CUDA library when the machine has at least 2 GPUs. A failure test checks that a rank that dies
before the exchange makes the surviving rank fail with an error instead of hanging.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
TINY = dict(vocab_size=256, embedding_dim=128, layer_count=2, head_count=4, kv_head_count=4, ffn_hidden=344,
            max_sequence_length=64)


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def full_batch():
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from projectai_b200 import _paihost as H
    r = H.PcgRng(7)
    ids = np.array([r.next_u32() % 256 for _ in range(4 * 33)], np.float32).reshape(4, 33)
    return np.ascontiguousarray(ids[:, :32]), np.ascontiguousarray(ids[:, 1:])


def make_trainer(H, be, world, seed=0):
    m = H.LlamaModel(be, H.ModelConfig(**TINY), seed=seed)
    tc = H.TrainingConfig(batch_size=4 // world, sequence_length=32, learning_rate=1e-3, weight_decay=0.1, max_steps=10,
                          gradient_checkpointing=True, warmup_steps=0)
    tr = H.Trainer(be, m, tc, 0.9, 0.95)
    tr.set_constant_lr(1e-3)
    return m, tr


def _gloo_rank(rank, world, port, out_dir, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from projectai_b200 import _paihost as H
    be = H.Backend(str(ROOT / "oracle" / "build" / "liboracle.so"), "oracle_", 0)
    m, tr = make_trainer(H, be, world)
    tr.world = world

    def allreduce(grads):
        for t in grads:
            host = torch.from_numpy(be.to_host(t).copy())
            dist.all_reduce(host)
            be.copy(be.from_host(host.numpy()), t)

    tr.set_allreduce(allreduce)
    x, y = full_batch()
    per = 4 // world
    status = "ok"
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the step")
        tr.step([x[rank * per:(rank + 1) * per].copy()], [y[rank * per:(rank + 1) * per].copy()])
    except Exception as e:  # a surviving rank must see its collective fail, not hang
        status = "error: " + type(e).__name__
    if status != "ok":
        np.savez(out_dir / f"rank{rank}.npz", status=status)
        return
    np.savez(out_dir / f"rank{rank}.npz", status=status,
             **{"p_" + n: be.to_host(p) for n, p in m.named_parameters()},
             **{"g_" + n: be.to_host(p.grad) for n, p in m.named_parameters() if p.grad is not None})
    if fail_rank < 0:
        dist.destroy_process_group()


def single_process_reference(lib, prefix):
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from projectai_b200 import _paihost as H
    be = H.Backend(str(lib), prefix, 0)
    m, tr = make_trainer(H, be, 1)
    x, y = full_batch()
    tr.step([x], [y])
    return ({n: be.to_host(p.grad) for n, p in m.named_parameters()}, {n: be.to_host(p) for n, p in m.named_parameters()})


def test_gloo_two_ranks_match_full_batch(tmp_path):
    port = free_port()
    mp.spawn(_gloo_rank, args=(2, port, tmp_path, -1), nprocs=2, join=True)
    ref_g, ref_p = single_process_reference(ROOT / "oracle" / "build" / "liboracle.so", "oracle_")
    r0 = np.load(tmp_path / "rank0.npz")
    r1 = np.load(tmp_path / "rank1.npz")
    assert str(r0["status"]) == "ok" and str(r1["status"]) == "ok"
    for n in ref_g:
        # rank grads after the exchange are the sum over ranks; AdamW divides by the world size
        np.testing.assert_array_equal(r0["g_" + n], r1["g_" + n])
        np.testing.assert_allclose(r0["g_" + n] / 2, ref_g[n], rtol=1e-4, atol=1e-6 * np.abs(ref_g[n]).max() + 1e-9,
                                   err_msg=n)
        np.testing.assert_array_equal(r0["p_" + n], r1["p_" + n])  # replicas stay identical
        # The first AdamW step moves each weight by lr·g/(|g|+eps); where g is at rounding-noise level its sign is
        # decided by summation order, so those elements are bounded by 2·lr (as in test_model_parity).
        noise = np.abs(ref_g[n]) < 1e-4 * np.abs(ref_g[n]).max()
        err = np.abs(r0["p_" + n].astype(np.float64) - ref_p[n])
        assert np.all(err[~noise] <= 1e-5 * np.abs(ref_p[n][~noise]) + 2e-6), n
        assert np.all(err[noise] <= 2e-3 + 1e-6), n


def test_dead_rank_fails_the_collective_instead_of_hanging(tmp_path):
    port = free_port()
    ctx = mp.start_processes(_gloo_rank, args=(2, port, tmp_path, 1), nprocs=2, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(120)
        assert not p.is_alive(), "a rank hung"
    r0 = np.load(tmp_path / "rank0.npz")
    assert str(r0["status"]).startswith("error"), str(r0["status"])


def _nccl_rank(rank, world, port, out_dir, zero1=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    pai = __graft_entry__.load_package()
    from projectai_b200 import _paihost as H
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", rank)
    uid = [be.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    be.nccl_init(uid[0], rank, world, 60000)
    m, tr = make_trainer(H, be, world)
    tr.zero1 = zero1
    x, y = full_batch()
    per = 4 // world
    tr.step([x[rank * per:(rank + 1) * per].copy()], [y[rank * per:(rank + 1) * per].copy()])
    tag = "zero1_" if zero1 else ""
    np.savez(out_dir / f"{tag}rank{rank}.npz", **{"p_" + n: be.to_host(p) for n, p in m.named_parameters()},
             **{"g_" + n: be.to_host(p.grad) for n, p in m.named_parameters()})
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_two_gpus_match_full_batch(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = free_port()
    mp.spawn(_nccl_rank, args=(2, port, tmp_path), nprocs=2, join=True)
    import __graft_entry__
    pai = __graft_entry__.load_package()
    ref_g, ref_p = single_process_reference(pai.CUDA_LIB_PATH, "pai_")
    r0 = np.load(tmp_path / "rank0.npz")
    r1 = np.load(tmp_path / "rank1.npz")
    for n in ref_g:
        np.testing.assert_array_equal(r0["g_" + n], r1["g_" + n])
        np.testing.assert_allclose(r0["g_" + n] / 2, ref_g[n], rtol=1e-4, atol=1e-4 * np.abs(ref_g[n]).max(), err_msg=n)
        np.testing.assert_array_equal(r0["p_" + n], r1["p_" + n])


def gloo_collectives(be, rank, world):
    """Sum-all-reduce, in-place reduce-scatter and in-place all-gather of backend tensors over the gloo group (rank
    r's shard of a flattened tensor is elements [r·n/W, (r+1)·n/W)), standing in for the backend's NCCL exchanges."""
    def allreduce(grads):
        for t in grads:
            host = torch.from_numpy(be.to_host(t).copy())
            dist.all_reduce(host)
            be.copy(be.from_host(host.numpy()), t)

    def shard_view(t):
        n = t.numel()
        return t.reshape([n]).slice(0, rank * (n // world), n // world)

    def reduce_scatter(grads):
        for t in grads:
            full = torch.from_numpy(be.to_host(t).copy()).reshape(-1)
            mine = torch.empty(full.numel() // world)
            dist.reduce_scatter_tensor(mine, full)
            be.copy(be.from_host(mine.numpy()), shard_view(t))

    def allgather(params):
        for p in params:
            mine = torch.from_numpy(be.to_host(shard_view(p)).copy())
            full = torch.empty(mine.numel() * world)
            dist.all_gather_into_tensor(full, mine)
            be.copy(be.from_host(full.numpy().reshape(be.to_host(p).shape)), p)

    return allreduce, reduce_scatter, allgather


# ---------------------------------------------------------------- ZeRO-1 (sharded AdamW state)
def _zero1_rank(rank, world, port, out_dir):
    """Two steps of the same data-parallel training, once with replicated AdamW (all-reduce) and once with ZeRO-1
    (reduce-scatter, AdamW on this rank's shard, all-gather), from the same initial weights."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from projectai_b200 import _paihost as H
    be = H.Backend(str(ROOT / "oracle" / "build" / "liboracle.so"), "oracle_", 0)

    allreduce, reduce_scatter, allgather = gloo_collectives(be, rank, world)

    x, y = full_batch()
    per = 4 // world
    out = {}
    for mode in ("replicated", "zero1"):
        m, tr = make_trainer(H, be, world)
        tr.world = world
        tr.rank = rank
        tr.set_allreduce(allreduce)
        if mode == "zero1":
            tr.zero1 = True
            tr.set_shard_exchange(reduce_scatter, allgather)
        for step in range(2):
            xs = np.roll(x, step, axis=0)[rank * per:(rank + 1) * per].copy()
            ys = np.roll(y, step, axis=0)[rank * per:(rank + 1) * per].copy()
            tr.step([xs], [ys])
        out.update({f"{mode}_p_{n}": be.to_host(p) for n, p in m.named_parameters()})
        out[f"{mode}_moments"] = np.array(tr.moment_elements())
        out["params"] = np.array(sum(be.to_host(p).size for _, p in m.named_parameters()))
    np.savez(out_dir / f"zero1_rank{rank}.npz", **out)
    dist.destroy_process_group()


def test_zero1_matches_replicated_adamw_bit_for_bit(tmp_path):
    port = free_port()
    mp.spawn(_zero1_rank, args=(2, port, tmp_path), nprocs=2, join=True)
    r0 = np.load(tmp_path / "zero1_rank0.npz")
    r1 = np.load(tmp_path / "zero1_rank1.npz")
    names = [k[len("replicated_p_"):] for k in r0.files if k.startswith("replicated_p_")]
    assert names
    for n in names:
        # the shards each rank updated, gathered, equal the replicated update bit for bit on both ranks
        np.testing.assert_array_equal(r0["zero1_p_" + n].view(np.uint32), r0["replicated_p_" + n].view(np.uint32), n)
        np.testing.assert_array_equal(r1["zero1_p_" + n].view(np.uint32), r0["zero1_p_" + n].view(np.uint32), n)
    # every parameter of the tiny model splits in two: each rank holds the moments of half of them
    assert int(r0["replicated_moments"]) == 2 * int(r0["params"])
    assert int(r0["zero1_moments"]) == int(r0["params"])


def _zero1_state_rank(rank, world, port, out_dir):
    """The checkpointed state of a ZeRO-1 run: its sharded moments gathered into the replicated layout, then applied
    to fresh trainers (sharded and replicated) that continue the run."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from projectai_b200 import _paihost as H
    be = H.Backend(str(ROOT / "oracle" / "build" / "liboracle.so"), "oracle_", 0)
    allreduce, reduce_scatter, allgather = gloo_collectives(be, rank, world)
    x, y = full_batch()
    per = 4 // world

    def batch(step):
        return ([np.roll(x, step, axis=0)[rank * per:(rank + 1) * per].copy()],
                [np.roll(y, step, axis=0)[rank * per:(rank + 1) * per].copy()])

    def trainer(zero1, seed=0):
        m, tr = make_trainer(H, be, world, seed)
        tr.world = world
        tr.rank = rank
        tr.set_allreduce(allreduce)
        if zero1:
            tr.zero1 = True
            tr.set_shard_exchange(reduce_scatter, allgather)
        return m, tr

    out = {}
    m_rep, t_rep = trainer(False)
    m_z, t_z = trainer(True)
    for step in range(2):
        t_rep.step(*batch(step))
        t_z.step(*batch(step))
    rep_items = t_rep.state_items()
    z_items = t_z.state_items()  # collective: both ranks gather the moment shards
    out["rep_names"] = np.array([n for n, _ in rep_items])
    out["z_names"] = np.array([n for n, _ in z_items])
    out.update({"rep_" + n: be.to_host(t) for n, t in rep_items})
    out.update({"z_" + n: be.to_host(t) for n, t in z_items})
    out["params"] = np.array(sum(be.to_host(p).size for _, p in m_z.named_parameters()))
    out["z_moments"] = np.array(t_z.moment_elements())

    # a sharded trainer from other weights takes the gathered state and continues in step with the original
    m_zr, t_zr = trainer(True, seed=1)
    t_zr.apply_state(z_items, 2)
    out["zr_moments"] = np.array(t_zr.moment_elements())
    m_rr, t_rr = trainer(False, seed=1)  # and so does a replicated one: the file is the same for both layouts
    t_rr.apply_state(z_items, 2)
    for tr in (t_z, t_zr, t_rr):
        tr.step(*batch(2))
    for tag, m in (("z3", m_z), ("zr3", m_zr), ("rr3", m_rr)):
        out.update({f"{tag}_p_" + n: be.to_host(p) for n, p in m.named_parameters()})

    if rank == 0:  # a sharded optimizer refuses moments that are not full-size (no collective on this path)
        bad = [(n, t.reshape([t.numel()]).slice(0, 0, 2) if n.startswith("opt.") else t) for n, t in z_items]
        try:
            t_zr.apply_state(bad, 2)
            out["bad"] = np.array("no error")
        except H.InvalidDataError as e:
            out["bad"] = np.array(str(e))
    np.savez(out_dir / f"zero1_state_rank{rank}.npz", **out)
    dist.destroy_process_group()


def test_zero1_checkpoint_state_gathers_and_restores_shards(tmp_path):
    """save_checkpoint's state under ZeRO-1 equals the replicated run's bit for bit (the moment shards are gathered
    into full-size tensors on every rank), and restoring it into sharded or replicated trainers continues the run
    exactly (Checkpointing.cs:103-142 layout; Optimizers.cs:81-123 update)."""
    port = free_port()
    mp.spawn(_zero1_state_rank, args=(2, port, tmp_path), nprocs=2, join=True)
    r0 = np.load(tmp_path / "zero1_state_rank0.npz")
    r1 = np.load(tmp_path / "zero1_state_rank1.npz")
    names = list(r0["rep_names"])
    assert list(r0["z_names"]) == names and list(r1["z_names"]) == names
    assert sum(n.startswith("opt.m::") for n in names) == sum(not n.startswith("opt.") for n in names)
    for n in names:
        for r in (r0, r1):
            np.testing.assert_array_equal(r["z_" + n].view(np.uint32), r0["rep_" + n].view(np.uint32), n)
    params = int(r0["params"])
    assert int(r0["z_moments"]) == params and int(r0["zr_moments"]) == params  # shards only: half of m and v each
    for r in (r0, r1):
        for k in r.files:
            if k.startswith("z3_p_"):
                n = k[len("z3_p_"):]
                np.testing.assert_array_equal(r["zr3_p_" + n].view(np.uint32), r[k].view(np.uint32), n)
                np.testing.assert_array_equal(r["rr3_p_" + n].view(np.uint32), r[k].view(np.uint32), n)
    assert "a sharded optimizer needs full-size moments" in str(r0["bad"]), str(r0["bad"])


def _train_loop_rank(rank, world, port, out_dir, accum):
    """Trainer.train under data parallelism with ZeRO-1 and `accum` micro-batches per step: rank r draws its rows
    from PCG stream (default + r) of the configured seed; the same draws stepped by hand give the same losses and
    weights."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from projectai_b200 import _paihost as H
    be = H.Backend(str(ROOT / "oracle" / "build" / "liboracle.so"), "oracle_", 0)
    allreduce, reduce_scatter, allgather = gloo_collectives(be, rank, world)
    data = np.random.RandomState(21).randint(0, 256, size=(9, 40))
    seqs = [[int(v) for v in row] for row in data]

    def trainer():
        m = H.LlamaModel(be, H.ModelConfig(**TINY), seed=0)
        tc = H.TrainingConfig(batch_size=2, sequence_length=32, learning_rate=1e-3, weight_decay=0.1, max_steps=2,
                              grad_accum=accum, gradient_checkpointing=True, warmup_steps=0, seed=77,
                              checkpoint_directory="")
        tr = H.Trainer(be, m, tc, 0.9, 0.95)
        tr.world = world
        tr.rank = rank
        tr.zero1 = True
        tr.set_allreduce(allreduce)
        tr.set_shard_exchange(reduce_scatter, allgather)
        return m, tr

    m1, t1 = trainer()
    report = t1.train(seqs)
    m2, t2 = trainer()
    stream = 0xDA3E39CB94B95BDB + rank if rank else 0xDA3E39CB94B95BDB
    rng = H.PcgRng(77, stream)
    manual, rows_seen = [], []
    for _ in range(2):
        xs, ys = [], []
        for _ in range(accum):
            rows = [rng.next_u32() % len(seqs) for _ in range(2)]
            rows_seen.append(rows)
            xs.append(np.array([seqs[r][:32] for r in rows], np.float32))
            ys.append(np.array([seqs[r][1:33] for r in rows], np.float32))
        manual.append(t2.step(xs, ys))
    np.savez(out_dir / f"train_rank{rank}.npz", losses=np.array(report["step_losses"], np.float32),
             manual=np.array(manual, np.float32), rows=np.array(rows_seen),
             **{"p_" + n: be.to_host(p) for n, p in m1.named_parameters()},
             **{"q_" + n: be.to_host(p) for n, p in m2.named_parameters()})
    dist.destroy_process_group()


@pytest.mark.parametrize("accum", [1, 2])
def test_train_loop_data_parallel_draws_per_rank_streams(tmp_path, accum):
    """Under data parallelism each rank's Trainer.train draws its own rows (rank 0 the reference's PcgRng(seed)
    sequence, rank r stream default + r), the ZeRO-1 exchanges run inside the loop (after the last micro-batch when a
    step accumulates two), and every rank ends with the weights a hand-driven run of the same draws reaches."""
    port = free_port()
    mp.spawn(_train_loop_rank, args=(2, port, tmp_path, accum), nprocs=2, join=True)
    r0 = np.load(tmp_path / "train_rank0.npz")
    r1 = np.load(tmp_path / "train_rank1.npz")
    assert not np.array_equal(r0["rows"], r1["rows"])  # the ranks see different rows
    for r in (r0, r1):
        assert np.array_equal(r["losses"], r["manual"])
        for k in r.files:
            if k.startswith("p_"):
                np.testing.assert_array_equal(r[k].view(np.uint32), r["q_" + k[2:]].view(np.uint32), k)
                np.testing.assert_array_equal(r[k].view(np.uint32), r0[k].view(np.uint32), k)  # replicas agree


def _zero1_files_rank(rank, world, port, out_dir):
    """Checkpoint files of a ZeRO-1 run through Trainer.train (rank 0 writes, both ranks gather), the same run
    replicated, and a restore of the ZeRO-1 file into fresh sharded trainers that continue the run."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    __graft_entry__.load_package()
    from projectai_b200 import _paihost as H
    be = H.Backend(str(ROOT / "oracle" / "build" / "liboracle.so"), "oracle_", 0)
    allreduce, reduce_scatter, allgather = gloo_collectives(be, rank, world)
    seqs = [[int(v) for v in row] for row in np.random.RandomState(22).randint(0, 256, size=(7, 40))]

    def trainer(zero1, seed, ckdir):
        m = H.LlamaModel(be, H.ModelConfig(**TINY), seed=seed)
        tc = H.TrainingConfig(batch_size=2, sequence_length=32, learning_rate=1e-3, weight_decay=0.1, max_steps=2,
                              gradient_checkpointing=True, warmup_steps=0, seed=5, checkpoint_every_steps=1,
                              checkpoint_directory=str(ckdir))
        tr = H.Trainer(be, m, tc, 0.9, 0.95)
        tr.world = world
        tr.rank = rank
        tr.set_allreduce(allreduce)
        if zero1:
            tr.zero1 = True
            tr.set_shard_exchange(reduce_scatter, allgather)
        return m, tr

    m_z, t_z = trainer(True, 0, out_dir / "z")
    t_z.train(seqs)
    m_r, t_r = trainer(False, 0, out_dir / "r")
    t_r.train(seqs)
    dist.barrier()  # rank 0's files are complete (the oracle writes them before save returns)
    m_x, t_x = trainer(True, 1, out_dir / "unused")
    assert t_x.restore(str(out_dir / "z" / "step-2.ckpt")) == 2
    x = np.array([seqs[rank][:32], seqs[rank + 2][:32]], np.float32)
    y = np.array([seqs[rank][1:33], seqs[rank + 2][1:33]], np.float32)
    t_z.step([x], [y])
    t_x.step([x], [y])
    np.savez(out_dir / f"files_rank{rank}.npz", moments=np.array(t_x.moment_elements()),
             **{"z_" + n: be.to_host(p) for n, p in m_z.named_parameters()},
             **{"x_" + n: be.to_host(p) for n, p in m_x.named_parameters()})
    dist.destroy_process_group()


def test_zero1_checkpoint_files_equal_the_replicated_run_and_resume(tmp_path):
    """Trainer.train under ZeRO-1 writes step-<n>.ckpt files byte-identical to the replicated run's (the moment shards
    gathered into the reference's layout, one writer), and sharded trainers restored from the last file continue the
    run bit for bit with shard-sized moments."""
    port = free_port()
    mp.spawn(_zero1_files_rank, args=(2, port, tmp_path), nprocs=2, join=True)
    for n in ("step-1.ckpt", "step-2.ckpt"):
        z, r = (tmp_path / "z" / n).read_bytes(), (tmp_path / "r" / n).read_bytes()
        assert z == r, n
    assert not (tmp_path / "unused").exists() or not any((tmp_path / "unused").iterdir())
    for rank in (0, 1):
        d = np.load(tmp_path / f"files_rank{rank}.npz")
        params = sum(d[k].size for k in d.files if k.startswith("z_"))
        assert int(d["moments"]) == params  # each rank holds half of m and half of v
        for k in d.files:
            if k.startswith("z_"):
                np.testing.assert_array_equal(d["x_" + k[2:]].view(np.uint32), d[k].view(np.uint32), k)


@pytest.mark.gpu
def test_nccl_zero1_two_gpus_matches_replicated(tmp_path):
    """ZeRO-1 over NCCL (in-place reduce-scatter, AdamW on the shard, in-place all-gather) gives the replicated
    update bit for bit: with two ranks both exchanges sum the same two values."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = free_port()
    mp.spawn(_nccl_rank, args=(2, port, tmp_path, False), nprocs=2, join=True)
    port = free_port()
    mp.spawn(_nccl_rank, args=(2, port, tmp_path, True), nprocs=2, join=True)
    for r in (0, 1):
        a = np.load(tmp_path / f"rank{r}.npz")
        b = np.load(tmp_path / f"zero1_rank{r}.npz")
        for k in a.files:
            if k.startswith("p_"):
                np.testing.assert_array_equal(a[k].view(np.uint32), b[k].view(np.uint32), k)


def _nccl_leave_rank(rank, world, port, out_dir):
    """Step 1 on both ranks; then rank 1 leaves (no further collective, nothing in flight) and rank 0 starts step 2.
    Rank 1 stays alive, its memory still mapped, until rank 0 has reported, then aborts its own communicator."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    pai = __graft_entry__.load_package()
    from projectai_b200 import _paihost as H
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", rank)
    uid = [be.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    be.nccl_init(uid[0], rank, world, 5000)  # every exchange is bounded by 5 s
    m, tr = make_trainer(H, be, world)
    x, y = full_batch()
    per = 4 // world
    xs, ys = x[rank * per:(rank + 1) * per].copy(), y[rank * per:(rank + 1) * per].copy()
    tr.step([xs], [ys])
    be.sync()
    dist.barrier()  # host-side (gloo): both ranks finished step 1, no kernel or collective in flight
    done = out_dir / "survivor_done"
    if rank == 1:
        for _ in range(1200):  # left the job; waits (at most 120 s) for the survivor's verdict
            if done.exists():
                break
            time.sleep(0.1)
        be.nccl_abort()
        return
    t0 = time.time()
    try:
        tr.step([xs], [ys])
        status = "ok"
    except Exception as e:  # the exchange with the departed peer must fail within the deadline
        status = f"error: {type(e).__name__}: {e}"
    np.savez(out_dir / "leave_rank0.npz", status=status, elapsed=time.time() - t0)
    done.touch()


@pytest.mark.gpu
def test_nccl_peer_leaving_between_steps_fails_within_the_deadline(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = free_port()
    ctx = mp.start_processes(_nccl_leave_rank, args=(2, port, tmp_path), nprocs=2, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(180)
        assert not p.is_alive(), "a rank hung"
    r0 = np.load(tmp_path / "leave_rank0.npz")
    status = str(r0["status"])
    assert status.startswith("error"), status
    assert "timeout" in status.lower() or "nccl" in status.lower(), status
    assert float(r0["elapsed"]) < 60.0, float(r0["elapsed"])
