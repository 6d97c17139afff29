"""The tensor-parallel decomposition of minq_tp_init, checked on the CPU with
two gloo ranks: each rank keeps its query / kv heads (q|k|v rows, o_proj
columns) and intermediate rows (gate/up rows, down_proj columns), runs the
reference's per-token steps (model.rs:273-318) with the oracle's ops, rank 0
adds the residual to its o_proj / down_proj partial, and an all-reduce sums
the ranks into x. The logits must match the oracle's single-rank forward.

The slicing mirrors minq_tp_init (csrc/model.cu): row ranges of the fused
q|k|v blocks, block-column ranges of o_proj / down_proj."""
import os

import numpy as np

CFG = dict(hidden_size=128, intermediate_size=256, n_layers=2, n_heads=4, n_kv_heads=2,
           head_dim=32, vocab_size=100, max_seq_len=16, rope_theta=1e6, rms_norm_eps=1e-6,
           has_qkv_bias=True, dtype="q8_0")
PROMPT = [3, 41, 7, 88, 19]
Q8, BB = 1, 36


def _model(orc):
    from minq_b200 import synth
    from minq_b200.minq_format import ModelConfig, quantize_tensor_rule
    cfg = ModelConfig(**CFG)
    t = {}
    for n, tag, s, d in synth.random_model_records(cfg, 7, qk_norm=True, with_bias=True):
        if n == "lm_head.weight":
            continue  # tied f32 lm_head
        t[n] = (Q8, s, orc.quantize(Q8, d)) if quantize_tensor_rule(n, s) else (tag, s, d)
    return t


def _rows(data, rows, cols, r0, r1):
    rb = cols // 32 * BB
    return np.ascontiguousarray(data.reshape(rows, rb)[r0:r1].reshape(-1))


def _cols(data, rows, cols, c0, c1):
    return np.ascontiguousarray(data.reshape(rows, cols // 32, BB)[:, c0 // 32:c1 // 32].reshape(-1))


def _rank_logits(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc
        t = _model(orc)
        H, I, nh, nkv, hd = (CFG[k] for k in ("hidden_size", "intermediate_size", "n_heads",
                                             "n_kv_heads", "head_dim"))
        eps, qd, kvd = CFG["rms_norm_eps"], nh * hd, nkv * hd
        nhl, nkvl, Il = nh // world, nkv // world, I // world
        q0, k0, i0 = rank * nhl * hd, rank * nkvl * hd, rank * Il
        cos, sin = orc.rope_tables(hd, CFG["max_seq_len"], CFG["rope_theta"])
        emb = t["model.embed_tokens.weight"][2].reshape(CFG["vocab_size"], H)
        kc = [[] for _ in range(CFG["n_layers"])]
        vc = [[] for _ in range(CFG["n_layers"])]

        def allreduce(v):
            ten = torch.from_numpy(v.copy())
            dist.all_reduce(ten)
            return ten.numpy().astype(np.float32)

        for pos, tok in enumerate(PROMPT):
            x = emb[tok].astype(np.float32).copy()
            for li in range(CFG["n_layers"]):
                p = f"model.layers.{li}."
                w = lambda n: t[p + n][2]
                xn = orc.rmsnorm(x, w("input_layernorm.weight"), eps)
                qv = orc.qmatvec(Q8, _rows(w("self_attn.q_proj.weight"), qd, H, q0, q0 + nhl * hd),
                                 nhl * hd, H, xn) + w("self_attn.q_proj.bias")[q0:q0 + nhl * hd]
                kv = orc.qmatvec(Q8, _rows(w("self_attn.k_proj.weight"), kvd, H, k0, k0 + nkvl * hd),
                                 nkvl * hd, H, xn) + w("self_attn.k_proj.bias")[k0:k0 + nkvl * hd]
                vv = orc.qmatvec(Q8, _rows(w("self_attn.v_proj.weight"), kvd, H, k0, k0 + nkvl * hd),
                                 nkvl * hd, H, xn) + w("self_attn.v_proj.bias")[k0:k0 + nkvl * hd]
                qv = orc.per_head_norm(qv, w("self_attn.q_norm.weight"), eps, hd)
                kv = orc.per_head_norm(kv, w("self_attn.k_norm.weight"), eps, hd)
                qv = orc.rope_apply_tables(cos, sin, qv, pos)
                kv = orc.rope_apply_tables(cos, sin, kv, pos)
                kc[li].append(kv)
                vc[li].append(vv)
                att = orc.attend(qv, np.concatenate(kc[li]), np.concatenate(vc[li]), pos + 1,
                                 nhl, nkvl, hd)
                o = orc.qmatvec(Q8, _cols(w("self_attn.o_proj.weight"), H, qd, q0, q0 + nhl * hd),
                                H, nhl * hd, att)
                x = allreduce(x + o if rank == 0 else o)
                xn = orc.rmsnorm(x, w("post_attention_layernorm.weight"), eps)
                g = orc.qmatvec(Q8, _rows(w("mlp.gate_proj.weight"), I, H, i0, i0 + Il), Il, H, xn)
                u = orc.qmatvec(Q8, _rows(w("mlp.up_proj.weight"), I, H, i0, i0 + Il), Il, H, xn)
                h = orc.silu(g) * u
                d = orc.qmatvec(Q8, _cols(w("mlp.down_proj.weight"), H, I, i0, i0 + Il), H, Il, h)
                x = allreduce(x + d if rank == 0 else d)
        logits = orc.matvec_f32(emb, orc.rmsnorm(x, t["model.norm.weight"][2], eps))
        q.put((rank, logits, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_split_matches_single_rank_on_cpu(orc):
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_logits, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        rank, logits, err = q.get(timeout=240)
        assert err is None, err
        got[rank] = logits
    for p in procs:
        p.join(timeout=60)
    t = _model(orc)
    om = orc.Model.from_tensors(CFG, t)
    ref = om.forward(PROMPT, om.new_cache())
    for rank in range(2):
        assert np.abs(got[rank] - ref).max() <= 1e-4 * max(1.0, float(np.abs(ref).max()))
    assert np.array_equal(got[0], got[1])  # the all-reduce leaves every rank the same x
