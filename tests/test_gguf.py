"""Ingest of ggml's interleaved blocks and of GGUF files (candelora_metal_kernels_b200.gguf).

CPU: a GGUF file written here (the format's published layout) is read back: metadata, tensor
directory and data offsets. GPU: the repack kernel (iq2_split_interleaved) inverts the
interleaving for every format, and a weight loaded from a GGUF file gives the same matmul as the
split tensors it was written from."""
import struct

import numpy as np
import pytest
import torch

import candelora_metal_kernels_b200 as c
from candelora_metal_kernels_b200 import gguf, synth

SPLIT = {16: (64, 2), 17: (64, 10), 22: (72, 10), 21: (104, 6)}  # ggml type -> (bytes, scale bytes)


def interleave(wb: np.ndarray, ws: np.ndarray, bpb: int, spb: int) -> np.ndarray:
    """Split tensors -> ggml blocks: d, the packed weights, then the remaining scale bytes."""
    nb = wb.size // bpb
    q, s = wb.reshape(nb, bpb), ws.reshape(nb, spb)
    return np.concatenate([s[:, :2], q, s[:, 2:]], axis=1).reshape(-1)


def _gguf_string(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, tensors, metadata=None, align=32):
    """Minimal GGUF v3 writer: tensors = [(name, shape ne-order, ggml type, bytes)]."""
    metadata = dict(metadata or {})
    head = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(metadata) + 1)
    kv = _gguf_string("general.alignment") + struct.pack("<II", 4, align)
    for k, v in metadata.items():
        kv += _gguf_string(k) + struct.pack("<I", 8) + _gguf_string(v)
    infos, data, off = b"", b"", 0
    for name, shape, gtype, raw in tensors:
        infos += _gguf_string(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        infos += struct.pack("<IQ", gtype, off)
        pad = (-len(raw)) % align
        data += raw + b"\0" * pad
        off += len(raw) + pad
    body = head + kv + infos
    body += b"\0" * ((-len(body)) % align)
    with open(path, "wb") as f:
        f.write(body + data)


def test_gguf_directory_roundtrip(tmp_path):
    n, k = 24, 512
    qs, sc = synth.iq2xxs_weights(n, k, seed=2)
    raw = interleave(qs.numpy(), sc.numpy(), 64, 2).tobytes()
    other = np.arange(10, dtype=np.float32).tobytes()
    path = tmp_path / "w.gguf"
    write_gguf(path, [("blk.0.ffn_up.weight", (k, n), 16, raw), ("norm", (10,), 0, other)],
               {"general.architecture": "llama"})
    r = gguf.GGUFReader(path)
    assert r.version == 3 and r.metadata["general.architecture"] == "llama"
    info = r.tensors["blk.0.ffn_up.weight"]
    assert info.shape == (k, n) and info.ggml_type == 16 and info.nbytes == len(raw)
    assert bytes(r.raw("blk.0.ffn_up.weight")) == raw
    assert r.tensors["norm"].nbytes is None
    with pytest.raises(ValueError):
        r.raw("norm")


def test_interleave_is_the_ggml_block_layout():
    # block_iq2_xxs: d (2 B) then qs (64 B); block_iq3_s: d, qs/qh/signs (104 B), scales (4 B)
    wb = np.arange(2 * 104, dtype=np.uint8)
    ws = (np.arange(2 * 6, dtype=np.uint8) + 200).astype(np.uint8)
    blocks = interleave(wb, ws, 104, 6).reshape(2, 110)
    assert list(blocks[1, :2]) == [206, 207] and list(blocks[1, 2:106]) == list(wb[104:])
    assert list(blocks[1, 106:]) == [208, 209, 210, 211]


@pytest.mark.gpu
@pytest.mark.parametrize("gtype", [16, 17, 22, 21])
@pytest.mark.parametrize("nblocks,offset", [(37, 0), (64 * 3 + 37, 0), (128, 0), (64 * 2 + 5, 2)])
def test_split_interleaved_inverts_the_blocks(gtype, nblocks, offset):
    """Fewer blocks than one 64-block chunk, whole chunks plus a tail, whole chunks only, and a
    source that is not 16-byte aligned (the byte-wise path)."""
    bpb, spb = SPLIT[gtype]
    rng = np.random.default_rng(gtype * 1000 + nblocks)
    wb, ws = rng.integers(0, 256, nblocks * bpb, dtype=np.uint8), rng.integers(0, 256, nblocks * spb, dtype=np.uint8)
    inter = interleave(wb, ws, bpb, spb)
    buf = torch.zeros(inter.size + offset, dtype=torch.uint8)
    buf[offset:] = torch.from_numpy(inter)
    blocks = buf.cuda()[offset:]
    got_b, got_s = gguf.split_interleaved(blocks, nblocks, gguf.GGML_TYPE[gtype])
    assert np.array_equal(got_b.cpu().numpy(), wb) and np.array_equal(got_s.cpu().numpy(), ws)


@pytest.mark.gpu
def test_gguf_weight_matmul(tmp_path):
    n, k = 1000, 1024
    qs, sc = synth.iq2xxs_weights(n, k, seed=4)
    path = tmp_path / "w.gguf"
    write_gguf(path, [("blk.3.attn_q.weight", (k, n), 16, interleave(qs.numpy(), sc.numpy(), 64, 2).tobytes())])
    wb, ws, out_dim, in_dim, variant = gguf.load_iq2_weight(path, "blk.3.attn_q.weight")
    assert (out_dim, in_dim, variant) == (n, k, c.Iq2MatmulVariant.Iq2Xxs)
    x = synth.activations(2, k, seed=5, device="cuda")
    assert torch.equal(c.iq2_xxs_matmul(x, wb, ws, n, k), c.iq2_xxs_matmul(x, qs.cuda(), sc.cuda(), n, k))
