"""Host-side tensor parallelism on CPU: the shard plan of the C ABI
(qwen_tp_plan, no GPU needed) and the exchange rules the decode kernel uses,
run as world-size-2 gloo ranks.

The kernel's rules, restated here and checked against the oracle:
  * a row-parallel projection (out_proj / o_proj over the rank's heads, down
    over its FFN columns) leaves one partial row per rank; every rank sums the
    partials in rank order and adds the residual, so all ranks hold the same
    hidden vector bit for bit, and it equals the unsharded product up to fp32
    rounding (exact in the int32 digit sums);
  * the head argmax takes each rank's (max, first index) of its vocab slice
    and keeps the largest value, the lowest index on ties (np.argmax's rule).
"""

import multiprocessing as mp
import socket

import numpy as np
import pytest

from oracle import golden_port as P

VOCAB = 248320


def _plan(rank, world):
    from qwen_fpga_b200 import api
    return api.tp_plan(rank, world)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_plan_partitions_every_dimension(world):
    plans = [_plan(r, world) for r in range(world)]
    # DeltaNet heads, OUT columns, FFN columns, vocab rows: contiguous and disjoint, covering all
    for key, total in (("dn_heads", 16), ("out_cols", 2048), ("ffn_cols", 3584), ("vocab", VOCAB)):
        lo = 0
        for p in plans:
            a, b = p[key]
            assert a == lo and b > a, (key, plans)
            lo = b
        assert lo == total, key
    for r, p in enumerate(plans):
        f0, f1 = p["ffn_cols"]
        assert f0 % 128 == 0 and f1 % 128 == 0           # whole 128-column MMA pieces
        o0, o1 = p["out_cols"]
        h0, h1 = p["dn_heads"]
        assert (o0, o1) == (h0 * 128, h1 * 128)          # the rank's DeltaNet heads x 128
        g0, g1 = p["kv_groups"]
        qh0, qh1 = o0 // 256, o1 // 256                  # its query heads (o_proj columns / 256)
        assert g0 <= qh0 // 4 and (qh1 - 1) // 4 < g1    # their KV groups are computed locally
        assert p["vocab"][0] % 128 == 0 and (p["vocab"][1] % 128 == 0)
    # every KV group is computed by some rank
    assert set().union(*(range(*p["kv_groups"]) for p in plans)) == {0, 1}


@pytest.mark.parametrize("world", [4, 8])
def test_kv_sequence_split_groups(world):
    """At 4 and 8 ranks each KV group is shared by ns = world / 2 ranks that are
    contiguous in rank order (the decode kernel's exchange addresses them as
    tp_rank - tp_rank % ns + j) and split its positions: the slices
    [j Tn / ns, (j + 1) Tn / ns) of those ranks tile [0, Tn) for every Tn,
    empty slices included when Tn < ns."""
    ns = world // 2
    plans = [_plan(r, world) for r in range(world)]
    for r, p in enumerate(plans):
        g0, g1 = p["kv_groups"]
        assert g1 - g0 == 1
        first = r - r % ns
        assert all(plans[q]["kv_groups"] == (g0, g1) for q in range(first, first + ns))
        assert all(plans[q]["kv_groups"] != (g0, g1) for q in range(world) if not first <= q < first + ns)
    for Tn in list(range(1, 40)) + [4097, 32769]:
        cover = []
        for j in range(ns):
            cover.extend(range(j * Tn // ns, (j + 1) * Tn // ns))
        assert cover == list(range(Tn))


@pytest.mark.parametrize("world,rank", [(3, 0), (16, 0), (2, 2), (2, -1)])
def test_tp_plan_rejects_bad_shards(world, rank):
    from qwen_fpga_b200 import api
    with pytest.raises(api.QwenError):
        api.tp_plan(rank, world)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    res = {"rank": rank}
    try:
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        from oracle import golden_port as Pg
        from qwen_fpga_b200 import api
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=60))
        plan = api.tp_plan(rank, world)
        rng = np.random.default_rng(11)                  # the same matrices on every rank
        out = {}
        for name, (K, key) in {"down": (3584, "ffn_cols"), "out": (2048, "out_cols")}.items():
            w = rng.integers(-127, 128, (1024, K), dtype=np.int8)
            x = rng.integers(-127, 128, K, dtype=np.int8)
            s = rng.uniform(1e-3, 1e-2, 1024).astype(np.float32)
            r = rng.standard_normal(1024).astype(np.float32)
            a, b = plan[key]
            acc = Pg.gemv_int32(w[:, a:b], x[a:b])       # this rank's exact partial digit sums
            part = torch.from_numpy(Pg.gemv_dequant(acc, 0.01, s))
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            tot = parts[0].clone()
            for p in parts[1:]:
                tot += p                                 # rank order
            h = (torch.from_numpy(r) + tot).numpy()
            full_acc = Pg.gemv_int32(w, x)
            acc_sum = [torch.from_numpy(Pg.gemv_int32(w[:, A:B], x[A:B]).astype(np.int64))
                       for A, B in (api.tp_plan(rr, world)[key] for rr in range(world))]
            out[name] = {
                "h": h,
                "exact": bool(np.array_equal(sum(t.numpy() for t in acc_sum), full_acc.astype(np.int64))),
                "ref": r + Pg.gemv_dequant(full_acc, 0.01, s),
            }
        # argmax exchange: planted ties across the two vocab slices
        logits = np.random.default_rng(5).standard_normal(VOCAB).astype(np.float32)
        lo0, hi0 = api.tp_plan(0, world)["vocab"]
        lo1, hi1 = api.tp_plan(world - 1, world)["vocab"]
        logits[hi0 - 7] = 9.0                            # in rank 0's slice
        logits[lo1 + 3] = 9.0                            # the same value in the last rank's
        lo, hi = plan["vocab"]
        i = int(np.argmax(logits[lo:hi]))
        mine = torch.tensor([float(logits[lo + i]), float(lo + i)], dtype=torch.float64)
        allp = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allp, mine)
        best = max(allp, key=lambda t: (t[0].item(), -t[1].item()))
        out["argmax"] = int(best[1].item())
        out["argmax_ref"] = int(np.argmax(logits))
        res.update(out)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        res["error"] = traceback.format_exc()
    q.put(res)


def test_tp_exchange_rules_on_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = []
    try:
        for _ in range(world):
            res.append(q.get(timeout=240))
    finally:
        for p in ps:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()   # this test's own child
    res.sort(key=lambda r: r["rank"])
    for r in res:
        assert "error" not in r, r["error"]
    for name in ("down", "out"):
        # every rank holds the same vector, bit for bit
        assert np.array_equal(res[0][name]["h"], res[1][name]["h"])
        # the shards' exact digit sums add up to the unsharded ones
        assert res[0][name]["exact"]
        ref = res[0][name]["ref"]
        err = np.abs(res[0][name]["h"] - ref).max() / np.abs(ref).max()
        assert err < 1e-6, err
    for r in res:
        assert r["argmax"] == r["argmax_ref"]            # the first index of the global max
