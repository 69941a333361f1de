"""Feature-cache reader (eacs_fc_*) against numpy on files written the way
the reference's npz_to_npy converter writes them (CPU; the device streaming
test is marked gpu)."""
import numpy as np
import pytest
import torch

from eacs_b200.feature_cache import FeatureCache, write_npy_pair


def _video(tmp_path, L=37, P=3, d=20, dtype=np.float16, ts_dtype=np.float64, stem="vid0"):
    rng = np.random.default_rng(L + P + d)
    feats = rng.standard_normal((L, P, d)).astype(dtype) if P else rng.standard_normal((L, d)).astype(dtype)
    ts = np.cumsum(rng.uniform(0.1, 1.0, L)).astype(ts_dtype)
    path = str(tmp_path / stem)
    np.save(path + ".npy", feats)
    np.save(path + ".ts.npy", ts)
    return path + ".npy", feats, ts


@pytest.mark.parametrize("P,dtype", [(3, np.float16), (1, np.float32), (0, np.float16)])
def test_read_matches_numpy(tmp_path, P, dtype):
    path, feats, ts = _video(tmp_path, P=P, dtype=dtype)
    with FeatureCache(path) as fc:
        assert (fc.L, fc.P, fc.d) == (37, max(P, 1), 20)
        ref = np.load(path, mmap_mode="r").reshape(37, max(P, 1), 20)
        assert np.array_equal(fc.read().numpy(), ref)
        assert np.array_equal(fc.read(5, 11).numpy(), ref[5:16])
        assert np.array_equal(fc.timestamps().numpy(), ts.astype(np.float32))
        with pytest.raises(RuntimeError, match="outside"):
            fc.read(30, 10)


def test_large_read_is_parallel_and_exact(tmp_path):
    path, feats, _ = _video(tmp_path, L=600, P=4, d=4096, stem="big")  # ~20 MB: several threads
    with FeatureCache(path) as fc:
        assert np.array_equal(fc.read(7, 500).numpy(), feats[7:507])


def test_rejects_bad_files(tmp_path):
    path, feats, ts = _video(tmp_path)
    np.save(str(tmp_path / "fort.npy"), np.asfortranarray(feats))
    np.save(str(tmp_path / "fort.ts.npy"), ts)
    with pytest.raises(RuntimeError, match="Fortran"):
        FeatureCache(str(tmp_path / "fort.npy"))
    np.save(str(tmp_path / "nots.npy"), feats)
    with pytest.raises(RuntimeError, match="cannot open"):
        FeatureCache(str(tmp_path / "nots.npy"))
    np.save(str(tmp_path / "short.npy"), feats)
    np.save(str(tmp_path / "short.ts.npy"), ts[:-1])
    with pytest.raises(RuntimeError, match="timestamps"):
        FeatureCache(str(tmp_path / "short.npy"))
    np.save(str(tmp_path / "int.npy"), feats.astype(np.int32))
    np.save(str(tmp_path / "int.ts.npy"), ts)
    with pytest.raises(RuntimeError, match="dtype"):
        FeatureCache(str(tmp_path / "int.npy"))
    (tmp_path / "junk.npy").write_bytes(b"not a numpy file at all")
    with pytest.raises(RuntimeError, match="not a .npy"):
        FeatureCache(str(tmp_path / "junk.npy"))


def _raw_npy(path, header: str, payload: bytes = b"\0" * 64):
    """A .npy file (format 1.0) with the given header dict text, and a
    matching timestamps file."""
    h = header.encode("latin1")
    h += b" " * ((-(10 + len(h) + 1)) % 64) + b"\n"
    with open(path, "wb") as f:
        f.write(b"\x93NUMPY\x01\x00" + len(h).to_bytes(2, "little") + h + payload)
    np.save(path[:-4] + ".ts.npy", np.zeros(4, np.float32))


def test_rejects_crafted_headers(tmp_path):
    """Shapes whose byte size wraps 64 bits, and a header cut off after a
    key, are rejected with an error (no read past the mapping, no abort)."""
    big = str(tmp_path / "big.npy")
    _raw_npy(big, "{'descr': '<f2', 'fortran_order': False, 'shape': (4, 4611686018427387904, 2), }")
    with pytest.raises(RuntimeError, match="too large|truncated"):
        FeatureCache(big)
    wrap = str(tmp_path / "wrap.npy")
    _raw_npy(wrap, "{'descr': '<f4', 'fortran_order': False, 'shape': (4, 1152921504606846976, 4), }")
    with pytest.raises(RuntimeError, match="too large|truncated"):
        FeatureCache(wrap)
    cut = str(tmp_path / "cut.npy")
    _raw_npy(cut, "{'descr': '<f2', 'fortran_order':" + " " * 40)
    with pytest.raises(RuntimeError, match="fortran_order|shape"):
        FeatureCache(cut)


def test_writer_round_trip(tmp_path):
    feats = np.arange(2 * 3 * 4, dtype=np.float16).reshape(2, 3, 4)
    path = write_npy_pair(str(tmp_path / "w"), feats, np.array([0.0, 0.5]))
    with FeatureCache(path) as fc:
        assert np.array_equal(fc.read().numpy(), feats)


@pytest.mark.gpu
def test_chunks_stream_to_device(tmp_path):
    path, feats, ts = _video(tmp_path, L=301, P=2, d=64, stem="dev")
    got, got_ts = [], []
    with FeatureCache(path) as fc:
        for l0, x, t in fc.chunks(64, "cuda:0"):
            assert x.is_cuda and x.shape[0] == min(64, 301 - l0)
            got.append((x.float() * 2).cpu())  # some work on the chunk
            got_ts.append(t.cpu())
    assert np.array_equal(torch.cat(got).numpy(), feats.astype(np.float32) * 2)
    assert np.array_equal(torch.cat(got_ts).numpy(), ts.astype(np.float32))
