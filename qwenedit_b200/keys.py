"""Prefix keys ("virtual ids") for the pools: one 63-bit int64 per token, chained so that equal ids imply an
equal prefix. Drop-in for ``multi_turn.cache.keys`` (keys.py:14-103): the id construction must stay
identical to the reference so both implementations address the same cached prefixes.

* digests are BLAKE2b-128 over length-prefixed parts (8-byte little-endian length, then the bytes);
* an id is the low 63 bits of a digest read little-endian;
* a text token's id digests (previous id, b"t", token as signed 8 bytes);
* the i-th token of an image block is splitmix64(base + i * 0x9E3779B97F4A7C15) masked to 63 bits, with
  base = id of digest(previous id, b"B", image content key [+ latent h, w for the DiT]).

Text chains and image blocks are computed by libqeb200 (native BLAKE2b, RFC 7693), one call per run; the
reference walks text tokens in a Python loop (keys.py:81-84). Root / content keys stay on hashlib (one digest
each).
"""

from __future__ import annotations

import hashlib
from collections.abc import Sequence

import numpy as np

from qwenedit_b200 import _lib

DIGEST = 16
MASK63 = (1 << 63) - 1


def _digest(*parts: bytes) -> bytes:
    h = hashlib.blake2b(digest_size=DIGEST)
    for part in parts:
        h.update(len(part).to_bytes(8, "little"))
        h.update(part)
    return h.digest()


def root_key(*identity: object) -> bytes:
    """Key root for one model identity (model path, quantisation, weights epoch ...)."""
    return _digest(b"root", repr(identity).encode())


def image_content_key(image) -> bytes:
    """Content key of a PIL image: mode, size and pixels."""
    return _digest(b"img", image.mode.encode(), repr(image.size).encode(), image.tobytes())


def latent_key(latent_id: str) -> bytes:
    return _digest(b"lat", latent_id.encode())


def _id(digest: bytes) -> int:
    return int.from_bytes(digest[:8], "little") & MASK63


def _i64(values) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(values, dtype=np.int64).reshape(-1))


def block_ids(prev: int, content: bytes, n: int) -> np.ndarray:
    """Ids of an n-token image block that follows id `prev`."""
    out = np.empty(n, np.int64)
    buf = np.frombuffer(content, dtype=np.uint8) if content else np.zeros(1, np.uint8)
    _lib.call("qe_keys_block_ids", int(prev), buf.ctypes.data, len(content), n, out.ctypes.data)
    return out


def text_chain(prev: int, tokens) -> np.ndarray:
    """Ids of text tokens chained from id `prev` (one native call for the whole run)."""
    toks = _i64(tokens)
    out = np.empty(len(toks), np.int64)
    if len(toks):
        _lib.call("qe_keys_text_chain", int(prev), toks.ctypes.data, len(toks), out.ctypes.data)
    return out


def text_id(prev: int, token: int) -> int:
    """Id of a text token that follows id `prev`."""
    return int(text_chain(prev, [token])[0])


def _text_chain(prev: int, tokens, out: np.ndarray) -> int:
    ids = text_chain(prev, list(tokens))
    out[:] = ids
    return int(ids[-1]) if len(ids) else prev


def virtual_ids(root: bytes, segments: Sequence[tuple[int, int, bool]], text_indices: Sequence[int],
                ids: Sequence[int], image_keys: Sequence[bytes], image_shapes: Sequence[tuple[int, int]]) -> np.ndarray:
    """Ids of the DiT prefix layout: text segments chain token by token, image segments are blocks keyed by
    content and latent shape (reference keys.py:61-87). Raises ValueError on a layout/shape mismatch."""
    total = segments[-1][1] if segments else 0
    out = np.empty(total, np.int64)
    prev, image = _id(root), 0
    for start, end, is_image in segments:
        if is_image:
            h, w = image_shapes[image]
            if end - start != h * w:
                raise ValueError("image segment length does not match its latent shape")
            content = image_keys[image] + np.asarray([h, w], np.int64).tobytes()
            out[start:end] = block_ids(prev, content, end - start)
            prev = int(out[end - 1])
            image += 1
        else:
            prev = _text_chain(prev, (ids[text_indices[p]] for p in range(start, end)), out[start:end])
    if image != len(image_keys):
        raise ValueError("image segments do not match the reference images")
    return out


def sequence_ids(root: bytes, token_ids: Sequence[int], image_runs: Sequence[tuple[int, int, bytes]]) -> np.ndarray:
    """Ids of the text-encoder sequence: tokens chain, each image-pad run is a content-keyed block
    (reference keys.py:90-103)."""
    out = np.empty(len(token_ids), np.int64)
    prev, position = _id(root), 0
    for start, end, key in sorted(image_runs):
        prev = _text_chain(prev, token_ids[position:start], out[position:start])
        out[start:end] = block_ids(prev, key, end - start)
        if end > start:
            prev = int(out[end - 1])
        position = end
    _text_chain(prev, token_ids[position:], out[position:])
    return out
