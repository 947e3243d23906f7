"""The GGUF reader and loader (crates/jevons-formats/src/gguf.rs).

CPU: the reference's own tests (gguf.rs:393-457: the sample file, its metadata and tensor, and
rejected magic / truncated data / truncated header), plus every rejection its reader makes.
GPU: a Q4_K layer tensor and a 3-D expert tensor loaded from a GGUF file dequantize bit-exactly.
"""
import struct

import numpy as np
import pytest

from jevons_kernels._lib import JkError
from jevons_kernels.gguf import Gguf


def s(text) -> bytes:
    raw = text.encode() if isinstance(text, str) else text
    return struct.pack("<Q", len(raw)) + raw


class Writer:
    """Builds GGUF bytes: metadata entries (key, kind, payload) and tensors (name, dims, type,
    data); tensor data is laid out in order at `alignment`, and the file ends with the last
    tensor's data."""

    def __init__(self, version=3, alignment=32):
        self.version, self.alignment = version, alignment
        self.kv, self.tensors = [], []

    def meta(self, key, kind, payload: bytes):
        self.kv.append(s(key) + struct.pack("<I", kind) + payload)
        return self

    def tensor(self, name, dims, type_, data: bytes, offset=None):
        self.tensors.append((name, dims, type_, data, offset))
        return self

    def build(self) -> bytes:
        out = b"GGUF" + struct.pack("<IQQ", self.version, len(self.tensors), len(self.kv)) + b"".join(self.kv)
        off, offsets = 0, []
        for _, _, _, data, fixed in self.tensors:
            offsets.append(off if fixed is None else fixed)
            off += (len(data) + self.alignment - 1) // self.alignment * self.alignment
        for (name, dims, type_, _, _), o in zip(self.tensors, offsets):
            out += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
            out += struct.pack("<IQ", type_, o)
        out += b"\0" * ((-len(out)) % self.alignment)
        for i, (_, _, _, data, _) in enumerate(self.tensors):
            out += data + (b"\0" * ((-len(data)) % self.alignment) if i + 1 < len(self.tensors) else b"")
        return out


def sample() -> bytes:
    """The reference test's file (gguf.rs:399-426): a.count = 7, a.names = ["x", "yz"], tensor
    w = F32 [2, 1] holding 1.5, -2.0."""
    w = Writer().meta("a.count", 4, struct.pack("<I", 7))
    w.meta("a.names", 9, struct.pack("<IQ", 8, 2) + s("x") + s("yz"))
    w.tensor("w", [2, 1], 0, struct.pack("<ff", 1.5, -2.0))
    return w.build()


def open_bytes(tmp_path, data: bytes, name="f.gguf") -> Gguf:
    p = tmp_path / name
    p.write_bytes(data)
    return Gguf.open(str(p))


def test_well_formed_files_expose_metadata_and_tensors(tmp_path):
    g = open_bytes(tmp_path, sample())
    assert g.u64("a.count") == 7
    assert g.get("a.names")[1] == "yz"
    assert g.read_f32("w").tolist() == [1.5, -2.0]
    info = g.tensor("w")
    assert info.dims == [2, 1] and info.kind == 0 and info.bytes == 8 and info.offset % 32 == 0


@pytest.mark.parametrize("name,cut", [("magic", "magic"), ("short", -4), ("header", 40)])
def test_truncated_or_corrupt_files_are_rejected(tmp_path, name, cut):
    good = sample()
    bad = b"GGUX" + good[4:] if cut == "magic" else good[:cut]
    with pytest.raises(JkError):
        open_bytes(tmp_path, bad, name)


def reject(tmp_path, data, text):
    with pytest.raises(JkError) as e:
        open_bytes(tmp_path, data)
    assert text in e.value.message, e.value.message


def test_rejections_carry_the_reference_messages(tmp_path):
    reject(tmp_path, b"GGUX" + sample()[4:], "Invalid GGUF file: bad magic")
    reject(tmp_path, Writer(version=1).build(), "Invalid GGUF file: unsupported version 1")
    reject(tmp_path, sample()[:40], "I/O error reading the model")
    reject(tmp_path, b"GGUF" + struct.pack("<IQQ", 3, 1 << 21, 0), "implausible header counts")
    reject(tmp_path, Writer().meta("k", 4, struct.pack("<I", 1)).meta("k", 4, struct.pack("<I", 2)).build(),
           "duplicate metadata key")
    reject(tmp_path, Writer().meta("k", 9, struct.pack("<IQ", 9, 1) + struct.pack("<IQ", 4, 0)).build(),
           "nested arrays are not supported")
    reject(tmp_path, Writer().meta("k", 7, b"\x02").build(), "invalid boolean")
    reject(tmp_path, Writer().meta("k", 13, b"").build(), "unknown metadata type 13")
    reject(tmp_path, Writer().meta("k", 8, struct.pack("<Q", (1 << 24) + 1)).build(), "string is too long")
    reject(tmp_path, Writer().meta("k", 8, s(b"\xff\xfe")).build(), "string is not UTF-8")
    reject(tmp_path, Writer().meta("k", 9, struct.pack("<IQ", 0, (1 << 26) + 1)).build(), "array is too long")
    reject(tmp_path, Writer().meta("general.alignment", 4, struct.pack("<I", 48)).build(), "invalid alignment")
    reject(tmp_path, Writer().tensor("t", [1, 1, 1, 1, 1], 0, b"\0" * 4).build(), "tensor t has 5 dimensions")
    reject(tmp_path, Writer().tensor("t", [100, 2], 12, b"\0" * 288).build(), "tensor t rows are not block aligned")
    reject(tmp_path, Writer().tensor("t", [256, 2], 12, b"\0" * 100).build(), "tensor t is out of bounds")
    reject(tmp_path, Writer().tensor("t", [1], 0, b"\0" * 4, offset=4).build(), "tensor t is out of bounds")
    reject(tmp_path, Writer().tensor("t", [1 << 40, 1 << 40], 0, b"").build(), "tensor t is too large")
    reject(tmp_path, Writer().tensor("t", [1], 0, b"\0" * 4).tensor("t", [1], 0, b"\0" * 4).build(),
           "duplicate tensor name")


def test_metadata_values_and_lookups(tmp_path):
    w = Writer(alignment=64).meta("general.alignment", 4, struct.pack("<I", 64))
    w.meta("i8", 1, struct.pack("<b", -3)).meta("u16", 2, struct.pack("<H", 65535))
    w.meta("f", 6, struct.pack("<f", 0.25)).meta("d", 12, struct.pack("<d", 1e-6)).meta("b", 7, b"\x01")
    w.meta("big", 10, struct.pack("<Q", 1 << 40)).meta("neg", 11, struct.pack("<q", -5))
    w.meta("name", 8, s("gemma")).meta("ids", 9, struct.pack("<IQ", 5, 3) + struct.pack("<iii", 1, -2, 3))
    w.tensor("x", [4], 0, struct.pack("<4f", 1, 2, 3, 4))
    w.tensor("q", [256, 2], 12, bytes(range(256)) + bytes(32))  # 2 Q4_K rows of raw bytes
    w.tensor("o", [4], 5, b"\0" * 4)  # an unsupported GGML type (I8): listed, not readable
    g = open_bytes(tmp_path, w.build())
    assert g.get("i8") == -3 and g.get("u16") == 65535 and g.get("b") is True
    assert g.f32("f") == 0.25 and g.get("d") == pytest.approx(1e-6, rel=1e-7)
    assert g.u64("big") == 1 << 40 and g.get("neg") == -5 and g.get("name") == "gemma"
    assert g.get("ids") == [1, -2, 3]
    with pytest.raises(JkError, match="neg is not an unsigned integer"):
        g.u64("neg")
    with pytest.raises(JkError, match="name is not a float"):
        g.f32("name")
    with pytest.raises(JkError, match="Missing GGUF metadata key nope"):
        g.u64("nope")
    with pytest.raises(JkError, match="Missing tensor nope"):
        g.tensor("nope")
    assert all(t.offset % 64 == 0 for t in g.tensors.values())
    q = g.tensor("q")
    assert q.bytes == 288 and g.read(q) == bytes(range(256)) + bytes(32)
    assert g.read_range(q, 250, 6) == bytes(range(250, 256))
    with pytest.raises(JkError, match="range is outside tensor q"):
        g.read_range(q, 200, 100)
    with pytest.raises(JkError, match="tensor o has unsupported type Other\\(5\\)"):
        g.read(g.tensor("o"))
    with pytest.raises(JkError, match="tensor q is not F32"):
        g.read_f32("q")
    assert g.read_f32("x").tolist() == [1, 2, 3, 4]


@pytest.mark.gpu
def test_weights_load_from_gguf_and_dequantize_exactly(gpu, tmp_path):
    from jevons_kernels import synth
    from jevons_kernels.gguf import load_qmatrix
    from oracle import oracle
    rng = np.random.default_rng(9)
    layer = synth.q4k_blocks(rng, 128, 512)
    experts = synth.q6k_blocks(rng, 3 * 64, 256)
    w = Writer().tensor("blk.0.ffn_up.weight", [512, 128], 12, layer.tobytes())
    w.tensor("blk.0.ffn_up_exps.weight", [256, 64, 3], 14, experts.tobytes())
    g = open_bytes(tmp_path, w.build())
    a = load_qmatrix(gpu, g, "blk.0.ffn_up.weight")
    assert (a.n, a.k, a.experts) == (128, 512, 1)
    got = a.dequantize().cpu().numpy().reshape(-1)
    assert np.array_equal(got.view(np.uint32), oracle.dequantize(oracle.Q4_K, layer).view(np.uint32))
    b = load_qmatrix(gpu, g, "blk.0.ffn_up_exps.weight")
    assert (b.n, b.k, b.experts) == (64, 256, 3)
    got = b.dequantize().cpu().numpy().reshape(-1)
    assert np.array_equal(got.view(np.uint32), oracle.dequantize(oracle.Q6_K, experts).view(np.uint32))
