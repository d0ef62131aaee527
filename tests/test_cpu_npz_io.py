"""The parallel `.npz` block reader against np.load (CPU only)."""
import zipfile

import numpy as np
import pytest

from synapcore_b200.npz_io import read_npz, read_npz_many


def _same(got, path):
    with np.load(path) as z:
        assert set(got) == set(z.files)
        for name in z.files:
            assert got[name].dtype == z[name].dtype and got[name].shape == z[name].shape
            assert np.array_equal(got[name], z[name])


def test_reads_fp16_and_int8_blocks_like_np_load(tmp_path):
    rng = np.random.default_rng(5)
    k = rng.standard_normal((2, 1, 4, 16, 128)).astype(np.float16)
    q = rng.integers(-127, 128, size=(2, 1, 4, 16, 128), dtype=np.int8)
    s = rng.random((2, 1, 4, 16, 1)).astype(np.float16)
    np.savez(tmp_path / "a.npz", k=k, v=-k)
    np.savez(tmp_path / "b.npz", kq=q, ks=s, vq=-q, vs=s)
    np.savez_compressed(tmp_path / "c.npz", k=k, v=k)  # deflated: np.load fallback
    np.savez(tmp_path / "d.npz", k=np.asfortranarray(k[0, 0]))  # Fortran order: fallback
    paths = [tmp_path / f"{n}.npz" for n in "abcd"]
    for got, p in zip(read_npz_many(paths), paths):
        _same(got, p)


def test_crc_mismatch_raises_like_np_load(tmp_path):
    k = np.arange(2 * 16 * 128, dtype=np.float16).reshape(2, 16, 128)
    np.savez(tmp_path / "a.npz", k=k)
    raw = bytearray((tmp_path / "a.npz").read_bytes())
    raw[len(raw) // 2] ^= 0x40
    (tmp_path / "bad.npz").write_bytes(bytes(raw))
    with pytest.raises(zipfile.BadZipFile):
        read_npz(tmp_path / "bad.npz")
    with pytest.raises(zipfile.BadZipFile):
        with np.load(tmp_path / "bad.npz") as z:
            z["k"]
