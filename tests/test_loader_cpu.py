"""The streaming loader's archive reader (no GPU): each ``.npy`` member of a saved index is parsed
from its header and read in chunks, with skips, exactly as ``np.load`` reads it whole."""

import zipfile

import numpy as np
import pytest

import maxsim_b200 as m
from maxsim_b200.loader import _Member


def _corpus(tmp_path, mode, seed=3):
    rng = np.random.default_rng(seed)
    lengths = rng.integers(0, 9, size=23)
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(offsets[-1]), 128)).astype(np.float32)
    idx = m.Index.from_embeddings([f"d{i}" for i in range(23)], docs, offsets, mode=mode)
    path = tmp_path / f"{mode}.npz"
    idx.save(path)
    return path


@pytest.mark.parametrize("mode", ["int4", "int4_per_token", "int4_residual"])
@pytest.mark.parametrize("compressed", [True, False])
def test_member_reader_matches_np_load(tmp_path, mode, compressed):
    path = _corpus(tmp_path, mode)
    with np.load(path) as data:
        arrays = {k: data[k] for k in data.files}
    if not compressed:
        path = tmp_path / "stored.npz"
        np.savez(path, **arrays)
    with zipfile.ZipFile(path) as archive:
        for name in ("int4_data", "int4_token_scale", "residual_int4_data", "doc_offsets"):
            if name not in arrays:
                continue
            ref = arrays[name]
            member = _Member(archive, name)
            assert member.shape == ref.shape and member.dtype == ref.dtype
            assert np.array_equal(member.read_array(), ref)
            member.close()
            if ref.ndim == 0 or ref.shape[0] < 4:
                continue
            # skip whole rows, then read the rest in odd-sized byte chunks
            member = _Member(archive, name)
            first = ref.shape[0] // 3
            member.skip(first * member.row_bytes)
            rest = np.ascontiguousarray(ref[first:]).reshape(-1).view(np.uint8)
            got = np.empty_like(rest)
            for lo in range(0, rest.size, 37):
                member.read_into(got[lo:lo + 37])
            assert np.array_equal(got, rest)
            member.close()


def test_member_reader_rejects_truncated_and_missing(tmp_path):
    path = _corpus(tmp_path, "int4")
    with zipfile.ZipFile(path) as archive:
        member = _Member(archive, "int4_data")
        too_many = np.empty(member.shape[0] * member.row_bytes + 1, np.uint8)
        with pytest.raises(ValueError, match="truncated"):
            member.read_into(too_many)
        member.close()
        with pytest.raises(KeyError, match="not a file"):
            _Member(archive, "no_such_array")


def test_uncompressed_save_round_trips(tmp_path):
    path = _corpus(tmp_path, "int4_per_token")
    idx = m.Index.load(path)
    stored = tmp_path / "stored.npz"
    idx.save(stored, compress=False)
    with zipfile.ZipFile(stored) as archive:
        assert all(info.compress_type == zipfile.ZIP_STORED for info in archive.infolist())
    again = m.Index.load(stored)
    assert again.doc_ids == idx.doc_ids
    assert np.array_equal(again.int4_packed.data, idx.int4_packed.data)
    assert np.array_equal(again.int4_packed.token_scale, idx.int4_packed.token_scale)


def test_package_imports_without_the_built_library(tmp_path):
    """A fresh checkout has no libmaxsim_b200.so yet: importing the package (and its build module)
    must work so the library can be built; only a call into the library fails."""
    import shutil
    import subprocess
    import sys
    from pathlib import Path

    src = Path(m.__file__).parent
    shutil.copytree(src, tmp_path / "maxsim_b200", ignore=shutil.ignore_patterns("*.so", "_build", "__pycache__"))
    code = ("import maxsim_b200, maxsim_b200.loader, maxsim_b200.build\n"
            "try:\n    maxsim_b200.loader._native()\nexcept ImportError as e:\n    print('missing:', e)\n")
    out = subprocess.run([sys.executable, "-c", code], cwd=tmp_path, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "missing:" in out.stdout and "no CPU fallback" in out.stdout
