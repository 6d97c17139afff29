"""Tensor-parallel decode (minq_tp_init: q|k|v rows and o_proj columns split
by head, gate/up rows and down_proj columns split by intermediate row, one
all-reduce after o_proj and after down_proj) on 2 GPUs, one process per GPU,
against the CPU oracle: logits max-abs < 1e-3, greedy tokens identical. Both
all-reduce paths: the one-shot peer-memory kernel (default) and NCCL
(MINQ_TP_NCCL=1). Needs two GPUs; skipped on one."""
import multiprocessing as mp

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(hidden_size=256, intermediate_size=512, n_layers=2, n_heads=4, n_kv_heads=2,
           head_dim=64, vocab_size=300, max_seq_len=64, rope_theta=1e6, rms_norm_eps=1e-6,
           has_qkv_bias=True, dtype="q8_0")
PROMPT = [5, 17, 230, 41, 99, 7]
NDEC = 8


def _records(orc):
    from minq_b200 import synth
    from minq_b200.minq_format import ModelConfig, quantize_tensor_rule
    cfg = ModelConfig(**CFG)
    out = []
    for n, t, s, d in synth.random_model_records(cfg, 31, qk_norm=True, with_bias=True):
        if n == "lm_head.weight":
            continue  # tied f32 lm_head (Qwen3)
        out.append((n, 1, s, orc.quantize(1, d)) if quantize_tensor_rule(n, s) else (n, t, s, d))
    return cfg, out


def _worker(rank, world, uid, q, nccl):
    try:
        import os
        os.environ["MINQ_TP_NCCL"] = "1" if nccl else "0"
        import torch
        torch.cuda.set_device(rank)
        import minq_b200 as mq
        from oracle import oracle as orc
        cfg, recs = _records(orc)
        model = mq.Model.from_tensors(cfg, recs)
        model.tp_init(rank, world, uid)
        cache = model.new_cache()
        tok, logits = model.forward_argmax(PROMPT, cache, logits=True)
        toks = [tok]
        for _ in range(NDEC):
            toks.append(model.forward_argmax([toks[-1]], cache))
        q.put((rank, logits, toks, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))


@pytest.mark.parametrize("nccl", [False, True], ids=["peer_allreduce", "nccl_allreduce"])
def test_tensor_parallel_two_gpus_matches_oracle(orc, nccl):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import minq_b200 as mq
    uid = mq.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, uid, q, nccl)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, logits, toks, err = q.get(timeout=300)
        assert err is None, err
        res[rank] = (logits, toks)
    for p in procs:
        p.join(timeout=60)
    cfg, recs = _records(orc)
    om = orc.Model.from_tensors(CFG, {n: (t, s, d) for n, t, s, d in recs})
    ref = om.forward(PROMPT, om.new_cache())
    ref_toks, _ = orc.greedy_generate(om, PROMPT, NDEC + 1)
    for rank in range(2):
        logits, toks = res[rank]
        assert np.abs(logits - ref).max() < 1e-3
        assert toks == ref_toks


CFG8 = dict(hidden_size=256, intermediate_size=2048, n_layers=2, n_heads=16, n_kv_heads=8,
            head_dim=64, vocab_size=300, max_seq_len=64, rope_theta=1e6, rms_norm_eps=1e-6,
            has_qkv_bias=True, dtype="q8_0")


def _worker_n(rank, world, uid, q):
    try:
        import os
        os.environ["MINQ_TP_NCCL"] = "0"
        import torch
        torch.cuda.set_device(rank)
        import minq_b200 as mq
        from oracle import oracle as orc
        cfg, recs = _records_cfg(orc, CFG8)
        model = mq.Model.from_tensors(cfg, recs)
        model.tp_init(rank, world, uid)
        cache = model.new_cache()
        tok, logits = model.forward_argmax(PROMPT, cache, logits=True)
        toks = [tok]
        from minq_b200 import _lib
        for i in range(NDEC):
            n0 = _lib.lib().minq_kernel_launches()
            toks.append(model.forward_argmax([toks[-1]], cache))
            if i == NDEC - 1:  # one launch per token: the decode megakernel ran
                torch.cuda.synchronize()
                launches = _lib.lib().minq_kernel_launches() - n0
        q.put((rank, logits, (toks, launches), None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))


def _records_cfg(orc, cfgd):
    from minq_b200 import synth
    from minq_b200.minq_format import ModelConfig, quantize_tensor_rule
    cfg = ModelConfig(**cfgd)
    out = []
    for n, t, s, d in synth.random_model_records(cfg, 37, qk_norm=True, with_bias=True):
        if n == "lm_head.weight":
            continue
        out.append((n, 1, s, orc.quantize(1, d)) if quantize_tensor_rule(n, s) else (n, t, s, d))
    return cfg, out


@pytest.mark.parametrize("world", [4, 8])
def test_tensor_parallel_four_and_eight_gpus_match_oracle(orc, world):
    """Eight kv heads split 4 or 8 ways (one or two kv heads and 2 or 4 query
    heads per rank, 512 or 256 intermediate rows), the decode megakernel's
    in-launch peer exchange on every rank, against the oracle."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import minq_b200 as mq
    uid = mq.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_n, args=(r, world, uid, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, logits, toks, err = q.get(timeout=300)
        assert err is None, err
        res[rank] = (logits, toks)
    for p in procs:
        p.join(timeout=60)
    cfg, recs = _records_cfg(orc, CFG8)
    om = orc.Model.from_tensors(CFG8, {n: (t, s, d) for n, t, s, d in recs})
    ref = om.forward(PROMPT, om.new_cache())
    ref_toks, _ = orc.greedy_generate(om, PROMPT, NDEC + 1)
    for rank in range(world):
        logits, (toks, launches) = res[rank]
        assert np.abs(logits - ref).max() < 1e-3
        assert toks == ref_toks
        assert launches == 1, launches
