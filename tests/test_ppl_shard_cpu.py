"""Perplexity data-sharded over ranks, checked on the CPU with two gloo ranks.

eval_ppl (ppl.rs:44-103) scores non-overlapping windows independently, so a
multi-GPU run gives each rank a contiguous run of whole windows (the token
slice starts on a window boundary) and combines the ranks' (nll sum, scored
count) with one all-reduce: mean_nll = sum / count. The ranks here run the
oracle's eval_ppl on their slices; the combined mean must equal the
single-rank eval_ppl of the whole sequence up to the order of the f64 sum,
and the counts exactly."""
import os

import numpy as np

from minq_b200.minq_format import ModelConfig

TINY = ModelConfig(64, 128, 2, 4, 4, 16, 128, 64, 10000.0, 1e-5, False, "f32")
N, CONTEXT, WORLD = 150, 16, 2  # 10 windows: 5 per rank, the last one 6 tokens


def _oracle_model():
    from minq_b200 import synth
    from oracle import oracle as orc
    recs = {n: (t, s, d) for n, t, s, d in synth.random_model_records(TINY, 21)}
    cfg = {k: getattr(TINY, k) for k in TINY.__dataclass_fields__}
    return orc, orc.Model.from_tensors(cfg, recs)


def _tokens():
    return np.random.default_rng(4).integers(0, TINY.vocab_size, N).astype(np.uint32)


def _rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _, om = _oracle_model()
        toks = _tokens()
        n_windows = -(-N // CONTEXT)
        per = -(-n_windows // world)
        mine = toks[rank * per * CONTEXT:(rank + 1) * per * CONTEXT]
        r = om.eval_ppl(mine, CONTEXT)
        part = torch.tensor([r["mean_nll"] * r["scored_positions"], float(r["scored_positions"])],
                            dtype=torch.float64)
        dist.all_reduce(part)
        q.put((rank, float(part[0]) / float(part[1]), int(part[1]), None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))
    finally:
        dist.destroy_process_group()


def test_ppl_window_sharding_matches_single_rank_on_cpu():
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        rank, mean, count, err = q.get(timeout=240)
        assert err is None, err
        got[rank] = (mean, count)
    for p in procs:
        p.join(timeout=60)
    _, om = _oracle_model()
    ref = om.eval_ppl(_tokens(), CONTEXT)
    for rank in range(WORLD):
        mean, count = got[rank]
        assert count == ref["scored_positions"]
        assert abs(mean - ref["mean_nll"]) <= 1e-12 * abs(ref["mean_nll"])
