"""Prefix keys: bit-identical to the reference's multi_turn/cache/keys.py (golden ids) and the reference's
key properties (tests/test_core.py:16-48)."""

import json
from pathlib import Path

import numpy as np
import pytest
from PIL import Image

from qwenedit_b200 import keys

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "keys.npz"), json.loads((GOLDEN / "keys.json").read_text())


def _images():
    a = Image.frombytes("RGB", (24, 16), bytes((np.arange(24 * 16 * 3) * 7 % 251).astype(np.uint8)))
    b = Image.frombytes("RGB", (24, 16), bytes((np.arange(24 * 16 * 3) * 11 % 253).astype(np.uint8)))
    return a, b


def test_roots_and_content_keys_match_reference(golden):
    _, meta = golden
    a, b = _images()
    assert keys.root_key("dit", "Qwen/Qwen-Image-2.1", None, None, None).hex() == meta["root"]
    assert keys.root_key("encoder", "Qwen2.5-VL", None).hex() == meta["encoder_root"]
    assert keys.image_content_key(a).hex() == meta["image_key_a"]
    assert keys.image_content_key(b).hex() == meta["image_key_b"]
    assert keys.latent_key("session/v3").hex() == meta["latent_key"]


@pytest.mark.parametrize("case", ["vids_one_image", "vids_two_images"])
def test_virtual_ids_match_reference(golden, case):
    arrays, meta = golden
    a, b = _images()
    ik = {"a": keys.image_content_key(a), "b": keys.image_content_key(b)}
    c = meta[case]
    root = bytes.fromhex(meta["root"])
    got = keys.virtual_ids(root, [tuple(s) for s in c["segments"]], c["text_indices"], meta["text_ids"],
                           [ik[k] for k in c["image_keys"]], [tuple(s) for s in c["image_shapes"]])
    assert got.dtype == np.int64
    np.testing.assert_array_equal(got, arrays[case])


def test_sequence_ids_match_reference(golden):
    arrays, meta = golden
    a, b = _images()
    ik = {"a": keys.image_content_key(a), "b": keys.image_content_key(b)}
    root = bytes.fromhex(meta["encoder_root"])
    runs = [(s, e, ik[k]) for s, e, k in meta["seq_two_runs"]]
    np.testing.assert_array_equal(keys.sequence_ids(root, meta["seq_tokens"], runs), arrays["seq_two_runs"])
    np.testing.assert_array_equal(keys.sequence_ids(root, meta["seq_tokens"][:50], []), arrays["seq_no_runs"])


SEGMENTS = ((0, 3, False), (3, 7, True), (7, 9, False))
TEXT_INDICES = [0, 1, 2, 3, 3, 3, 3, 4, 5]


def _vids(ids, image=b"img1"):
    return keys.virtual_ids(b"root", SEGMENTS, TEXT_INDICES, ids, [image], [(2, 2)])


def test_virtual_ids_share_head_and_split_at_first_difference():
    a, b = _vids([10, 11, 12, 99, 20, 21]), _vids([10, 11, 12, 99, 30, 31])
    assert (a[:7] == b[:7]).all() and a[7] != b[7] and a[8] != b[8]
    assert len(set(a.tolist())) == len(a)


def test_image_block_matches_whole_or_not_at_all():
    a, c = _vids([10, 11, 12, 99, 20, 21]), _vids([10, 11, 12, 99, 20, 21], b"img2")
    assert (a[:3] == c[:3]).all() and not (a[3:7] == c[3:7]).any() and not (a[7:] == c[7:]).any()


def test_layout_errors_raise():
    with pytest.raises(ValueError):
        keys.virtual_ids(b"r", ((0, 5, True),), [], [], [b"x"], [(2, 2)])
    with pytest.raises(ValueError):
        keys.virtual_ids(b"r", ((0, 2, False),), [0, 1], [5, 6], [b"x"], [])


def test_native_blake2b_matches_hashlib():
    import ctypes
    import hashlib

    from qwenedit_b200 import _lib

    rng = np.random.default_rng(0)
    for n in (0, 1, 41, 127, 128, 129, 255, 256, 257, 1000, 4096):
        msg = rng.integers(0, 256, size=n, dtype=np.uint8).tobytes()
        out = (ctypes.c_uint8 * 16)()
        buf = np.frombuffer(msg, np.uint8) if n else np.zeros(1, np.uint8)
        _lib.call("qe_blake2b16", buf.ctypes.data, n, ctypes.addressof(out))
        assert bytes(out) == hashlib.blake2b(msg, digest_size=16).digest(), n


def test_native_text_chain_matches_the_digest_definition():
    import hashlib

    def ref_text_id(prev, token):  # keys.py:57-58 written out with hashlib
        h = hashlib.blake2b(digest_size=16)
        for part in (prev.to_bytes(8, "little"), b"t", int(token).to_bytes(8, "little", signed=True)):
            h.update(len(part).to_bytes(8, "little"))
            h.update(part)
        return int.from_bytes(h.digest()[:8], "little") & ((1 << 63) - 1)

    prev = 12345
    toks = [0, 1, -5, 2**40, 151643, 7]
    want = []
    for t in toks:
        prev = ref_text_id(prev, t)
        want.append(prev)
    np.testing.assert_array_equal(keys.text_chain(12345, toks), np.array(want, np.int64))
