"""`.minq` writer / reader in Python, byte-compatible with format.rs.

Layout (format.rs:3-15): magic "MINQ0001" | u32 LE config-JSON length |
config JSON (serde_json of ModelConfig) | records until EOF, each
u32 name_len | name | u8 tag (0 f32, 1 q8_0, 2 q4_0) | u8 ndim |
ndim x u64 shape | u64 data length | data.

The config JSON is written exactly as serde_json writes ModelConfig
(model.rs:29-45): fields in declaration order, compact separators, integers
in decimal and the two f32 fields in ryu's shortest round-trip notation, so a
file written here is byte-identical to the reference's `write_minq`.
The quantize selection rule and sorted record order of `minq quantize`
(main.rs:303,340-352) are in `quantize_tensor_rule` / `write_minq`.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, asdict

import numpy as np

MAGIC = b"MINQ0001"          # format.rs:30
LEGACY_MAGIC = b"MINFER01"   # format.rs:35
TAG_F32, TAG_Q8_0, TAG_Q4_0 = 0, 1, 2
BLOCK_SIZE = 32
BLOCK_BYTES = {TAG_Q8_0: 36, TAG_Q4_0: 20}
DTYPE_TAGS = {"f32": TAG_F32, "q8_0": TAG_Q8_0, "q4_0": TAG_Q4_0}


@dataclass
class ModelConfig:
    """model.rs:29-45 (field order is the serialisation order)."""

    hidden_size: int
    intermediate_size: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab_size: int
    max_seq_len: int
    rope_theta: float
    rms_norm_eps: float
    has_qkv_bias: bool
    dtype: str

    def __post_init__(self):
        # rope_theta / rms_norm_eps are f32 in the reference
        self.rope_theta = float(np.float32(self.rope_theta))
        self.rms_norm_eps = float(np.float32(self.rms_norm_eps))

    def to_json(self) -> str:
        parts = []
        for k, v in asdict(self).items():
            if isinstance(v, bool):
                s = "true" if v else "false"
            elif k in ("rope_theta", "rms_norm_eps"):
                s = format_f32(v)
            elif isinstance(v, str):
                s = json.dumps(v)
            else:
                s = str(int(v))
            parts.append(f'"{k}":{s}')
        return "{" + ",".join(parts) + "}"

    @classmethod
    def from_json(cls, text: str) -> "ModelConfig":
        d = json.loads(text)
        vals = {}
        for k in cls.__dataclass_fields__:
            if k not in d:
                raise ValueError(f"json error: missing field `{k}`")
            vals[k] = d[k]
        vals["rope_theta"] = float(np.float32(vals["rope_theta"]))
        vals["rms_norm_eps"] = float(np.float32(vals["rms_norm_eps"]))
        return cls(**vals)


def format_f32(v: float) -> str:
    """serde_json / ryu `format32` of an f32: shortest round-trip digits laid
    out as integer (`1000000.0`), decimal (`12.34`, `0.000001`) or exponent
    (`1e-7`, `1.234e33`) notation."""
    f = np.float32(v)
    if not np.isfinite(f):
        return "null"
    neg = bool(np.signbit(f))
    if f == 0:
        return "-0.0" if neg else "0.0"
    sci = np.format_float_scientific(abs(f), unique=True, trim="-")
    mant, exp = sci.split("e")
    # mant has one digit before the point: value = 0.d1d2.. * 10^(exp+1)
    digits = mant.replace(".", "").rstrip("0") or "0"
    length = len(digits)
    k = int(exp) - (length - 1)  # value = int(digits) * 10^k
    kk = length + k
    if 0 <= k and kk <= 13:
        s = digits + "0" * k + ".0"
    elif 0 < kk <= 13:
        s = digits[:kk] + "." + digits[kk:]
    elif -6 < kk <= 0:
        s = "0." + "0" * (-kk) + digits
    elif length == 1:
        s = digits + "e" + str(kk - 1)
    else:
        s = digits[0] + "." + digits[1:] + "e" + str(kk - 1)
    return ("-" if neg else "") + s


def quantize_tensor_rule(name: str, shape) -> bool:
    """main.rs:343-346: quantize 2-D `.weight` tensors (not the embedding)
    whose columns are a multiple of the block size."""
    return (name.endswith(".weight") and "embed_tokens" not in name and len(shape) == 2
            and shape[1] % BLOCK_SIZE == 0)


def write_minq_header(f, config: ModelConfig) -> None:  # format.rs:64-70
    cfg = config.to_json().encode()
    f.write(MAGIC)
    f.write(struct.pack("<I", len(cfg)))
    f.write(cfg)


def write_minq_record(f, name: str, tag: int, shape, data) -> None:  # format.rs:74-99
    nb = name.encode()
    f.write(struct.pack("<I", len(nb)))
    f.write(nb)
    f.write(struct.pack("<BB", tag, len(shape)))
    for d in shape:
        f.write(struct.pack("<Q", int(d)))
    buf = np.ascontiguousarray(data)
    if tag == TAG_F32:
        buf = buf.astype("<f4", copy=False)
    else:
        buf = buf.astype(np.uint8, copy=False)
    f.write(struct.pack("<Q", buf.nbytes))
    f.write(buf.tobytes())


def write_minq(path, config: ModelConfig, records) -> None:
    """records: iterable of (name, tag, shape, data), written in the given
    order (`minq quantize` writes them sorted by name, main.rs:303)."""
    with open(path, "wb") as f:
        write_minq_header(f, config)
        for name, tag, shape, data in records:
            write_minq_record(f, name, tag, shape, data)


class FormatError(ValueError):
    pass


def read_minq(path):
    """format.rs:149-277 with the same length checks; returns (config, list of
    (name, tag, shape, np.ndarray))."""
    file_len = os.path.getsize(path)
    pos = 0

    def take(n, what):
        nonlocal pos
        if pos + n > file_len:
            raise FormatError(f"{path}: {what} claims {n} bytes at offset {pos}, "
                              f"file is {file_len} bytes")
        pos += n

    with open(path, "rb") as f:
        take(8, "magic")
        magic = f.read(8)
        if magic not in (MAGIC, LEGACY_MAGIC):
            raise FormatError(f"{path}: not a .minq/.minfer file (bad magic)")
        take(4, "config length")
        (cfg_len,) = struct.unpack("<I", f.read(4))
        take(cfg_len, "config json")
        config = ModelConfig.from_json(f.read(cfg_len).decode())
        records = []
        while True:
            first = f.read(1)
            if not first:
                break
            take(4, "tensor name length")
            (name_len,) = struct.unpack("<I", first + f.read(3))
            take(name_len, "tensor name")
            name = f.read(name_len).decode()
            take(2, "tensor tag/ndim")
            tag, ndim = struct.unpack("<BB", f.read(2))
            take(8 * ndim, "tensor shape")
            shape = list(struct.unpack(f"<{ndim}Q", f.read(8 * ndim)))
            numel = 1
            for d in shape:
                numel *= d
            if numel >= 2 ** 64:
                raise FormatError(f"tensor `{name}`: shape {shape} overflows usize")
            take(8, "tensor data length")
            (data_len,) = struct.unpack("<Q", f.read(8))
            if tag == TAG_F32:
                expected = numel * 4
            elif tag in (TAG_Q8_0, TAG_Q4_0):
                if ndim != 2:
                    raise FormatError(f"quantized tensor `{name}` must be 2-D, got {shape}")
                if shape[1] % BLOCK_SIZE:
                    raise FormatError(f"quantized tensor `{name}`: cols {shape[1]} not block-aligned")
                expected = shape[0] * (shape[1] // BLOCK_SIZE) * BLOCK_BYTES[tag]
            else:
                raise FormatError(f"tensor `{name}`: unknown storage tag {tag}")
            if expected >= 2 ** 64:
                raise FormatError(f"tensor `{name}`: byte count overflows")
            if data_len != expected:
                raise FormatError(f"tensor `{name}`: data length {data_len} != shape-derived {expected}")
            take(data_len, "tensor data")
            raw = f.read(data_len)
            arr = (np.frombuffer(raw, dtype="<f4").reshape(shape) if tag == TAG_F32
                   else np.frombuffer(raw, dtype=np.uint8))
            records.append((name, tag, shape, arr))
    return config, records
