""".minq format: the Python writer/reader (minq_b200.minq_format) against
format.rs's layout and hardening tests (format.rs:311-434), read back by the
oracle's C++ reader. CPU only."""
import struct

import numpy as np
import pytest

from minq_b200.minq_format import (LEGACY_MAGIC, MAGIC, ModelConfig, TAG_F32, TAG_Q8_0,
                                   FormatError, format_f32, quantize_tensor_rule, read_minq,
                                   write_minq)


def make_config():  # format.rs:284
    return ModelConfig(64, 128, 2, 4, 2, 16, 128, 64, 10000.0, 1e-5, False, "q8_0")


def sample_records(orc):  # format.rs:301
    dense = np.array([[1, 2, 3], [4, 5, 6]], dtype=np.float32)
    w = (np.arange(4 * 64, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    q = orc.quantize_q8_0(w)
    return [("dense.weight", TAG_F32, [2, 3], dense), ("quant.weight", TAG_Q8_0, [4, 64], q)]


def test_config_json_is_serde_layout():
    cfg = ModelConfig(896, 4864, 24, 14, 2, 64, 151936, 4096, 1e6, 1e-6, True, "q8_0")
    assert cfg.to_json() == (
        '{"hidden_size":896,"intermediate_size":4864,"n_layers":24,"n_heads":14,'
        '"n_kv_heads":2,"head_dim":64,"vocab_size":151936,"max_seq_len":4096,'
        '"rope_theta":1000000.0,"rms_norm_eps":0.000001,"has_qkv_bias":true,"dtype":"q8_0"}')


@pytest.mark.parametrize("v,s", [(1e6, "1000000.0"), (1e-6, "0.000001"), (1e-5, "0.00001"),
                                 (10000.0, "10000.0"), (5e5, "500000.0"), (1e-7, "1e-7"),
                                 (0.1, "0.1"), (123.456, "123.456"), (1.5e30, "1.5e30"),
                                 (0.0, "0.0"), (-2.5, "-2.5")])
def test_format_f32_ryu(v, s):
    assert format_f32(v) == s


def test_minq_file_roundtrip(tmp_path, orc):  # format.rs:312
    p = tmp_path / "m.minq"
    recs = sample_records(orc)
    write_minq(p, make_config(), recs)
    raw = p.read_bytes()
    assert raw[:8] == MAGIC
    cfg, back = read_minq(p)
    assert cfg == make_config()
    for (n1, t1, s1, d1), (n2, t2, s2, d2) in zip(recs, back):
        assert (n1, t1, list(s1)) == (n2, t2, list(s2))
        assert np.array_equal(np.asarray(d1).reshape(-1).view(np.uint8),
                              np.asarray(d2).reshape(-1).view(np.uint8))
    n = np.zeros(1, dtype=np.uint64)
    assert orc.lib().orc_read_minq_count(str(p).encode(), n.ctypes.data) == 0
    assert int(n[0]) == 2


def test_legacy_minfer_magic_is_accepted(tmp_path, orc):  # format.rs:332
    p = tmp_path / "m.minfer"
    write_minq(p, make_config(), sample_records(orc))
    raw = bytearray(p.read_bytes())
    raw[:8] = LEGACY_MAGIC
    p.write_bytes(bytes(raw))
    cfg, back = read_minq(p)
    assert cfg == make_config() and len(back) == 2


def test_rejects_bad_magic(tmp_path):  # format.rs:353
    p = tmp_path / "bad.bin"
    p.write_bytes(b"NOTMINFER junk")
    with pytest.raises(FormatError):
        read_minq(p)


def crafted(tmp_path, tag, record: bytes):  # format.rs:363
    cfg = make_config().to_json().encode()
    p = tmp_path / f"crafted_{tag}.minq"
    p.write_bytes(MAGIC + struct.pack("<I", len(cfg)) + cfg + record)
    return p


CRAFTED = {
    # format.rs:387 name_len = u32::MAX with nothing behind it
    "huge_name_len": struct.pack("<I", 0xFFFFFFFF),
    # format.rs:394 f32 [1] with u64::MAX data length
    "huge_data_len": struct.pack("<I", 1) + b"a" + bytes([0, 1]) + struct.pack("<Q", 1)
    + struct.pack("<Q", 2 ** 64 - 1),
    # format.rs:407 f32 [2, 3] declares 8 data bytes
    "shape_data_mismatch": struct.pack("<I", 1) + b"w" + bytes([0, 2]) + struct.pack("<QQ", 2, 3)
    + struct.pack("<Q", 8) + bytes(8),
    # format.rs:422 [u64::MAX, 2] overflows the element count
    "shape_overflow": struct.pack("<I", 3) + b"big" + bytes([0, 2])
    + struct.pack("<QQ", 2 ** 64 - 1, 2) + struct.pack("<Q", 16) + bytes(16),
    # unknown storage tag / misaligned quantized cols
    "unknown_tag": struct.pack("<I", 1) + b"t" + bytes([7, 1]) + struct.pack("<QQ", 1, 4) + bytes(4),
    "q_cols_misaligned": struct.pack("<I", 1) + b"q" + bytes([1, 2]) + struct.pack("<QQ", 1, 33)
    + struct.pack("<Q", 36) + bytes(36),
    "truncated": struct.pack("<I", 1) + b"a" + bytes([0]),
}


@pytest.mark.parametrize("tag", sorted(CRAFTED))
def test_rejects_malformed_records(tmp_path, orc, tag):  # format.rs:386-434
    p = crafted(tmp_path, tag, CRAFTED[tag])
    with pytest.raises(FormatError):
        read_minq(p)
    n = np.zeros(1, dtype=np.uint64)
    assert orc.lib().orc_read_minq_count(str(p).encode(), n.ctypes.data) != 0


def test_quantize_selection_rule():  # main.rs:343-346
    assert quantize_tensor_rule("model.layers.0.mlp.up_proj.weight", [8, 64])
    assert not quantize_tensor_rule("model.embed_tokens.weight", [8, 64])
    assert not quantize_tensor_rule("model.layers.0.input_layernorm.weight", [64])
    assert not quantize_tensor_rule("model.layers.0.self_attn.q_proj.bias", [64])
    assert not quantize_tensor_rule("x.weight", [8, 33])


def _lib_load(path):
    import ctypes as C
    from minq_b200 import _lib
    L = _lib.lib()
    h = C.c_void_p()
    st = L.minq_model_load(str(path).encode(), C.byref(h))
    if st == _lib.OK:
        L.minq_model_free(h)
    return st, L.minq_last_error().decode()


@pytest.mark.parametrize("tag", sorted(CRAFTED))
def test_library_loader_rejects_malformed_records(tmp_path, mq, tag):  # format.rs:386-434
    """The product loader (mapped file, indexed in place) refuses the same
    records before it touches a device."""
    from minq_b200 import _lib
    st, msg = _lib_load(crafted(tmp_path, tag, CRAFTED[tag]))
    assert st == _lib.ERR_FORMAT, msg


def test_library_loader_reads_a_valid_file_up_to_the_device(tmp_path, mq, orc):
    """A valid file is indexed and handed to the uploader: on a machine
    without a GPU the load stops there with a device error (no CPU path)."""
    from minq_b200 import _lib
    import torch
    p = tmp_path / "m.minq"
    write_minq(p, make_config(), sample_records(orc))
    st, msg = _lib_load(p)
    if torch.cuda.is_available():
        assert st in (_lib.OK, _lib.ERR_SHAPE, _lib.ERR_MODEL), msg
    else:
        assert st == _lib.ERR_CUDA and "no CUDA device" in msg, msg
    st, msg = _lib_load(tmp_path / "missing.minq")
    assert st == _lib.ERR_IO and "cannot open" in msg
