"""Multi-rank host logic of the whole-sequence sharding, on CPU with gloo
(world size 2): plan broadcast and agreement, coverage of every token, the
gather back to global order, and detection of a failed rank by timeout."""

import datetime
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, q):
    try:
        import torch
        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5 if mode == "fail" else 60))
        from scree_b200 import shard, workloads

        lengths = workloads.cfg4_lengths()
        offs = np.concatenate([[0], np.cumsum(lengths)])
        plan = shard.plan_shards(lengths, world)
        if mode == "disagree" and rank == 1:
            plan = [plan[1], plan[0]]
        if mode == "fail" and rank == 1:
            raise SystemExit(0)  # this rank leaves before the first collective
        try:
            plan = shard.broadcast_plan(plan)
        except RuntimeError as e:
            # A peer that disagrees, or one that is gone (gloo raises on the
            # closed connection or after the process-group timeout).
            q.put((rank, "plan-mismatch" if "differs" in str(e) else "error", str(e)[:200]))
            return
        mine = shard.local_shard(offs, plan, rank)
        # Every rank "computes" on its rows: here, the global row index itself.
        vals = torch.as_tensor(mine.rows, dtype=torch.float64).reshape(-1, 1) * 2.0
        if mode == "fail":
            try:
                shard.gather_to_rank0(vals, mine, int(offs[-1]))
                q.put((rank, "no-error", ""))
            except Exception as e:  # the missing rank must surface as an error
                q.put((rank, "error", type(e).__name__))
            return
        if mode == "ok_plan":  # row lists derived from the plan: only values are sent
            out = shard.gather_to_rank0(vals, mine, int(offs[-1]), plan=plan, global_offsets=offs)
        elif mode == "gplan":  # one message per sequence into rank 0's output slices
            outs = shard.GatherPlan(plan, offs, rank, torch.device("cpu")).run([vals, vals * 3])
            out = None
            if rank == 0:
                assert torch.equal(outs[1], outs[0] * 3)
                out = outs[0]
        else:
            out = shard.gather_to_rank0(vals, mine, int(offs[-1]))
        if rank == 0:
            ok = torch.equal(out[:, 0], torch.arange(int(offs[-1]), dtype=torch.float64) * 2.0)
            q.put((rank, "gathered", ok))
        else:
            q.put((rank, "sent", out is None))
        dist.destroy_process_group()
    except BaseException:
        q.put((rank, "exception", traceback.format_exc()))


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    out = []
    while not q.empty():
        out.append(q.get())
    return sorted(out, key=lambda t: t[0])


def test_plan_covers_and_balances():
    from scree_b200 import shard, workloads

    lengths = workloads.cfg4_lengths()
    offs = np.concatenate([[0], np.cumsum(lengths)])
    for world in (1, 2, 4, 8):
        plan = shard.plan_shards(lengths, world)
        assert sorted(i for p in plan for i in p) == list(range(len(lengths)))
        assert shard.imbalance(lengths, plan) < 1.02
        rows = np.concatenate([shard.local_shard(offs, plan, r).rows for r in range(world)])
        assert np.array_equal(np.sort(rows), np.arange(offs[-1]))


def test_head_group_plan_covers_every_head_once_and_balances():
    """Splitting the heavy sequences by head groups removes the one-long-sequence
    cap: every config at 1-8 ranks is within 3% of perfect balance, where
    whole-sequence sharding is off by 2x for cfg2 / cfg5 at 8 ranks."""
    from scree_b200 import shard, workloads

    for name in ("cfg2", "cfg4", "cfg5"):
        cfg = workloads.attn_config(name)
        lengths, H = list(cfg.lengths), cfg.heads
        for world in (1, 2, 4, 8):
            plan = shard.plan_units(lengths, world, H, max_groups=16)
            cover = np.zeros((len(lengths), H), dtype=np.int64)
            for part in plan:
                for u in part:
                    assert 0 <= u.h0 < u.h1 <= H and H % u.heads == 0
                    cover[u.seq, u.h0:u.h1] += 1
            assert (cover == 1).all(), (name, world)
            assert shard.units_imbalance(lengths, plan) < 1.03, (name, world)
        if name in ("cfg2", "cfg5"):
            assert shard.imbalance(lengths, shard.plan_shards(lengths, 8)) > 1.9
        # The default keeps every unit at half the heads or more.
        assert all(u.heads >= H // 2 for part in shard.plan_units(lengths, 8, H) for u in part)
        groups = shard.units_by_heads(shard.plan_units(lengths, 8, H, max_groups=16)[0])
        assert all(all(u.heads == hs for u in us) for hs, us in groups.items())


def test_two_ranks_gather_global_order():
    res = _run("ok")
    assert [r[1] for r in res] == ["gathered", "sent"], res
    assert res[0][2] is True and res[1][2] is True


@pytest.mark.parametrize("mode", ["ok", "ok_plan", "gplan"])
def test_three_ranks_gather_point_to_point(mode):
    """Ranks 1 and 2 send to rank 0 only; rank 0 rebuilds global order, with the
    row lists sent or derived from the plan."""
    res = _run(mode, world=3)
    assert [r[1] for r in res] == ["gathered", "sent", "sent"], res
    assert all(r[2] is True for r in res), res


def test_two_ranks_detect_plan_disagreement():
    """Both ranks, rank 0 included (its own plan matches itself), raise the
    same mismatch error instead of one rank proceeding into the next collective."""
    res = _run("disagree")
    assert len(res) == 2 and all(r[1] == "plan-mismatch" for r in res), res


def test_missing_rank_is_an_error_not_a_hang():
    res = _run("fail", timeout=90)
    assert res and res[0][0] == 0 and res[0][1] in ("error", "exception"), res
