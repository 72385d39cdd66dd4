"""PBTQW25 v1 container: writer for seeded synthetic Qwen2.5-0.5B images.

The layout follows docs/PBTQW25-v1.md and model.rs:245-287,810-833 of
sulewicz/promptboot: a 256-byte header, seven 64-byte section entries, a
291-entry tensor directory (96 bytes each) and the tensor data, every section
and tensor 64-byte aligned, tensors back to back in id order.  The real
checkpoint is not available here, so the weights are random with the shapes and
dtypes of the frozen schema:

* Q4_0 tensors: per 32-block binary16 scale |N(0, 0.02)| / 8, nibbles uniform
  0..15 (low nibbles are elements 0..15, high nibbles 16..31);
* f32 biases N(0, 0.02), norm weights 1.0;
* tensor 290 (the Q8_0 lm_head): the reference's Q8_0 quantizer
  (fp32_sse2.rs:945-983) applied to the dequantized token embedding (tensor 0),
  so input and output embeddings stay tied as in the source model.

One numpy Generator(PCG64(seed)) draws, in tensor-id order, for every Q4_0
tensor first the scales then the nibbles, and for every bias its values.
Tokenizer sections are zero-filled (layout-only images).
"""
from __future__ import annotations

import hashlib
import os
import pathlib
import struct
import tempfile

import numpy as np

MODEL_BYTES = 426_762_944
VOCAB = 151_936
SECTION_OFFSETS = [704, 608_512, 1_981_312, 2_133_248, 3_949_952, 3_952_512, 3_980_480]
SECTION_LENGTHS = [607_748, 1_372_758, 151_936, 1_816_644, 2_509, 27_936, 422_782_464]
SECTION_COUNTS = [151_937, 1_372_758, 151_936, 151_387, 2_509, 291, 422_782_464]
SECTION_TYPES = [1, 2, 2, 3, 2, 4, 2]
SOURCE_HASH = bytes.fromhex("7671c0c304e6ce5a7fc577bcb12aba01e2c155cc2efd29b2213c95b18edaf6ed")
TENSOR_DIR = SECTION_OFFSETS[5]
TENSOR_DATA = SECTION_OFFSETS[6]

F32, Q4_0, Q8_0 = 1, 2, 3


def expected_tensor(tid: int):
    """model.rs:810-833: (layer, role, dtype, rank, dims)."""
    if tid == 0:
        return 0xFFFF, 1, Q4_0, 2, (896, 151_936, 1, 1)
    if tid == 289:
        return 0xFFFF, 2, F32, 1, (896, 1, 1, 1)
    if tid == 290:
        return 0xFFFF, 3, Q8_0, 2, (896, 151_936, 1, 1)
    layer, slot = (tid - 1) // 12, (tid - 1) % 12
    role = 10 + slot
    table = {0: (F32, 1, (896, 1, 1, 1)), 1: (Q4_0, 2, (4864, 896, 1, 1)),
             2: (Q4_0, 2, (896, 4864, 1, 1)), 3: (Q4_0, 2, (896, 4864, 1, 1)),
             4: (F32, 1, (896, 1, 1, 1)), 5: (F32, 1, (128, 1, 1, 1)),
             6: (Q4_0, 2, (896, 128, 1, 1)), 7: (Q4_0, 2, (896, 896, 1, 1)),
             8: (F32, 1, (896, 1, 1, 1)), 9: (Q4_0, 2, (896, 896, 1, 1)),
             10: (F32, 1, (128, 1, 1, 1)), 11: (Q4_0, 2, (896, 128, 1, 1))}
    dtype, rank, dims = table[slot]
    return layer, role, dtype, rank, dims


def tensor_bytes(tid: int) -> int:
    _, _, dtype, _, dims = expected_tensor(tid)
    n = dims[0] * dims[1] * dims[2] * dims[3]
    return n * 4 if dtype == F32 else n // 32 * (18 if dtype == Q4_0 else 34)


def tensor_offsets():
    offsets, at = [], TENSOR_DATA
    for tid in range(291):
        offsets.append(at)
        at += tensor_bytes(tid)
    assert at == MODEL_BYTES
    return offsets


def layer_tensor(layer: int, role: int) -> int:
    """model.rs:673-720 (tensor_for)."""
    return 1 + layer * 12 + (role - 10)


def _q4_blocks(rng: np.random.Generator, nblocks: int) -> np.ndarray:
    scales = (np.abs(rng.standard_normal(nblocks) * 0.02) / 8.0).astype(np.float16)
    nib = rng.integers(0, 16, size=(nblocks, 32), dtype=np.uint8)
    out = np.empty((nblocks, 18), dtype=np.uint8)
    out[:, :2] = scales.view(np.uint8).reshape(nblocks, 2)
    out[:, 2:] = nib[:, :16] | (nib[:, 16:] << 4)
    return out


def dequantize_q4_rows(blocks: np.ndarray) -> np.ndarray:
    """fp32_sse2.rs:897-922 for [rows][blocks][18] -> f32 [rows][blocks*32]."""
    d = blocks[..., :2].copy().view(np.float16)[..., 0].astype(np.float32)
    packed = blocks[..., 2:]
    q = np.concatenate([(packed & 15).astype(np.int16) - 8, (packed >> 4).astype(np.int16) - 8],
                       axis=-1).astype(np.float32)
    return (d[..., None] * q).reshape(blocks.shape[0], -1)


def quantize_q8_rows(x: np.ndarray) -> np.ndarray:
    """fp32_sse2.rs:945-983 vectorised: f32 [rows][K] -> [rows][K/32][34] blocks."""
    rows, k = x.shape
    xb = x.reshape(rows, k // 32, 32).astype(np.float32)
    amax = np.abs(xb).max(axis=-1)
    d = amax / np.float32(127.0)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0.0), np.float32(1.0) / d).astype(np.float32)
    v = xb * inv[..., None]
    half = np.where(np.signbit(v), np.float32(-0.5), np.float32(0.5)).astype(np.float32)
    q = np.trunc(v + half).astype(np.int32).astype(np.int8)
    out = np.empty((rows, k // 32, 34), dtype=np.uint8)
    out[..., :2] = d.astype(np.float16).view(np.uint8).reshape(rows, k // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out


def synthesize(seed: int = 0) -> np.ndarray:
    """Build the whole image in memory (426,762,944 bytes, uint8)."""
    rng = np.random.default_rng(seed)
    img = np.zeros(MODEL_BYTES, dtype=np.uint8)
    offsets = tensor_offsets()
    for tid in range(290):
        layer, role, dtype, rank, dims = expected_tensor(tid)
        at, n = offsets[tid], tensor_bytes(tid)
        if dtype == Q4_0:
            nblocks = dims[0] * dims[1] // 32
            img[at:at + n] = _q4_blocks(rng, nblocks).reshape(-1)
        elif role in (15, 18, 20):
            vals = (rng.standard_normal(dims[0]) * 0.02).astype(np.float32)
            img[at:at + n] = vals.view(np.uint8)
        else:
            img[at:at + n] = np.ones(dims[0], dtype=np.float32).view(np.uint8)
    emb = img[offsets[0]:offsets[0] + tensor_bytes(0)].reshape(VOCAB, 28, 18)
    out = img[offsets[290]:offsets[290] + tensor_bytes(290)].reshape(VOCAB, 28, 34)
    for r0 in range(0, VOCAB, 8192):
        r1 = min(VOCAB, r0 + 8192)
        out[r0:r1] = quantize_q8_rows(dequantize_q4_rows(emb[r0:r1]))
    _write_directories(img, offsets)
    return img


def _write_directories(img: np.ndarray, offsets) -> None:
    buf = memoryview(img)
    for tid in range(291):
        layer, role, dtype, rank, dims = expected_tensor(tid)
        at = TENSOR_DIR + tid * 96
        n = tensor_bytes(tid)
        digest = hashlib.sha256(buf[offsets[tid]:offsets[tid] + n]).digest()
        entry = struct.pack("<IHHII4IQQ32s16x", tid, layer, role, dtype, rank, *dims,
                            offsets[tid], n, digest)
        img[at:at + 96] = np.frombuffer(entry, dtype=np.uint8)
    for ordinal in range(7):
        off, ln = SECTION_OFFSETS[ordinal], SECTION_LENGTHS[ordinal]
        digest = hashlib.sha256(buf[off:off + ln]).digest()
        entry = struct.pack("<IIQQQ32s", ordinal + 1, SECTION_TYPES[ordinal],
                            SECTION_COUNTS[ordinal], off, ln, digest)
        img[256 + ordinal * 64:256 + ordinal * 64 + 64] = np.frombuffer(entry, dtype=np.uint8)
    header = struct.pack("<8sIIIIIIIIIIIIIIIIIIQQQQQQ", b"PBTQW25\0", 1, 256, 0x01020304, 7, 291,
                         151_936, 151_387, 32_768, 24, 896, 4864, 14, 2, 64, 151_645, 151_643,
                         151_643, 0, 428_730_208, MODEL_BYTES, 256, 448, 5_947_744, 422_782_464)
    img[:len(header)] = np.frombuffer(header, dtype=np.uint8)
    img[128:160] = np.frombuffer(SOURCE_HASH, dtype=np.uint8)
    img[160:192] = np.frombuffer(hashlib.sha256(buf[256:]).digest(), dtype=np.uint8)


def cache_path(seed: int = 0) -> pathlib.Path:
    base = os.environ.get("PB_MODEL_CACHE") or tempfile.gettempdir()
    return pathlib.Path(base) / f"promptboot_b200_synthetic_seed{seed}.pbtqw25"


def load_or_synthesize(seed: int = 0) -> np.ndarray:
    """The seeded image, cached on disk between processes."""
    path = cache_path(seed)
    if path.exists() and path.stat().st_size == MODEL_BYTES:
        return np.fromfile(path, dtype=np.uint8)
    img = synthesize(seed)
    tmp = path.with_suffix(f".tmp{os.getpid()}")
    img.tofile(tmp)
    os.replace(tmp, path)
    return img


def tensor_view(img: np.ndarray, tid: int) -> np.ndarray:
    """Raw bytes of tensor `tid` read through the image's own directory."""
    off, n = struct.unpack_from("<QQ", img, TENSOR_DIR + tid * 96 + 32)
    return img[off:off + n]
