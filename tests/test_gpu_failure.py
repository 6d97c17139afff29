"""Failure detection without a GPU fault.

Device side: every wait in the decode megakernel (ring slots, grid barrier,
per-head attention merge) is bounded (1 s of %globaltimer). The test moves
one wait's target out of reach from the host (minq_debug_inject_timeout, a
target nothing will reach), checks that the step reports the timeout
(MinqError Timeout, error.rs-style status MINQ_ERR_TIMEOUT) and that the model
stays usable: a fresh cache then decodes exactly like the oracle.

Host side: minq_tp_init meets the other ranks under a deadline
(MINQ_TP_INIT_TIMEOUT_S); a rank whose peer never joins gets MinqError Nccl
instead of blocking. Only NCCL's bootstrap waits there (no GPU kernel runs),
in a child process.
"""
import multiprocessing as mp
import os
import time

import numpy as np
import pytest

from minq_b200.minq_format import ModelConfig, quantize_tensor_rule
from minq_b200 import synth

pytestmark = pytest.mark.gpu


def _tiny(orc):
    cfg = ModelConfig(256, 512, 2, 8, 2, 64, 300, 64, 1e6, 1e-6, False, "q4_0")
    recs = []
    for n, t, s, d in synth.random_model_records(cfg, 41, qk_norm=True):
        if n == "lm_head.weight":
            continue  # tied f32 lm_head: the decode megakernel's shape
        recs.append((n, 2, s, orc.quantize(2, d)) if quantize_tensor_rule(n, s) else (n, t, s, d))
    return cfg, recs


@pytest.mark.parametrize("what", [0, 1], ids=["attention_merge_wait", "grid_barrier_wait"])
def test_megakernel_wait_times_out_and_recovers(mq, orc, what):
    from minq_b200 import _lib, api, MinqError
    cfg, recs = _tiny(orc)
    model = mq.Model.from_tensors(cfg, recs)
    om = orc.Model.from_tensors({k: getattr(cfg, k) for k in cfg.__dataclass_fields__},
                                {n: (t, s, d) for n, t, s, d in recs})
    prompt = [3, 77, 150, 9]
    cache = model.new_cache()
    model.forward(prompt, cache)
    L = _lib.lib()
    assert L.minq_debug_inject_timeout(model._h, what) == _lib.OK, L.minq_last_error()
    t0 = time.perf_counter()
    with pytest.raises(MinqError) as ei:
        model.forward([5], cache)
    el = time.perf_counter() - t0
    assert ei.value.status == _lib.ERR_TIMEOUT, ei.value
    assert el < 30.0
    # the model is usable again: a fresh cache decodes like the oracle
    cache2 = model.new_cache()
    logits = model.forward(prompt, cache2)
    ref = om.forward(prompt, om.new_cache())
    assert np.abs(logits - ref).max() < 1e-3
    got = []
    api.Engine(model, api.Sampler.greedy()).generate(prompt, 6, got.append)
    ref_toks, _ = orc.greedy_generate(om, prompt, 6)
    assert got == ref_toks


def _lonely_rank(uid, q):
    try:
        os.environ["MINQ_TP_INIT_TIMEOUT_S"] = "4"
        import torch
        torch.cuda.set_device(0)
        import minq_b200 as mq
        from minq_b200 import MinqError, _lib
        from oracle import oracle as orc
        cfg, recs = _tiny(orc)
        model = mq.Model.from_tensors(cfg, recs)
        t0 = time.perf_counter()
        try:
            model.tp_init(0, 2, uid)  # rank 1 never joins
            q.put(("joined", None, time.perf_counter() - t0))
        except MinqError as e:
            q.put(("error", (e.status, str(e)), time.perf_counter() - t0))
    except Exception as e:  # reported to the parent
        q.put(("exception", repr(e), 0.0))


def test_tp_init_times_out_when_a_rank_never_joins(mq):
    from minq_b200 import _lib
    uid = mq.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(uid, q))
    p.start()
    kind, info, el = q.get(timeout=240)
    p.join(timeout=60)
    assert kind == "error", (kind, info)
    status, msg = info
    assert status == _lib.ERR_NCCL, msg
    assert "did not all join" in msg, msg
    assert el < 60.0
