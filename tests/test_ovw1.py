"""The OVW1 reader of the C ABI (ovb_ovw1_*) on the CPU: files written by
ovnative_b200.ovw1.write (and the reference's own minimal test file,
cpp/tests/test_gemm.cpp:354-405) read back tensor for tensor; every check of
ov::WeightFile::Open (cpp/src/core/weight_file.cpp:124-206) rejects the file
it should with the reference's message; CRC32 agrees with zlib's."""
from __future__ import annotations

import struct
import zlib

import numpy as np
import pytest

import oracle as O
from ovnative_b200 import ovw1

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


def sample_tensors(rng):
    Wnk = rng.integers(-127, 128, size=(96, 64), dtype=np.int8)
    Wkn = rng.integers(-127, 128, size=(64, 40), dtype=np.int8)
    return [
        ("model.norm.weight", rng.standard_normal(64).astype(np.float32), 0, None),
        ("layers.0.q_proj.weight", Wnk, 0, (rng.random(96) * 1e-3).astype(np.float32)),
        ("layers.0.o_proj.weight", Wkn, 1, (rng.random(40) * 1e-3).astype(np.float32)),
        ("conv.weight", rng.standard_normal((4, 3, 5)).astype(np.float16), 0, None),
        ("positions", np.arange(7, dtype=np.int64), 0, None),
        ("scalar", np.array(2.5, dtype=np.float32), 0, None),
    ]


def test_round_trip(repo_tmp):
    rng = np.random.default_rng(1)
    ts = sample_tensors(rng)
    p = str(repo_tmp / "m.ovw")
    ovw1.write(p, ts, flags=3)
    with ovw1.OVW1File(p) as f:
        assert len(f) == len(ts)
        assert f.names() == [t[0] for t in ts]
        h = f.header()
        assert h["dtype_mode"] == 1 and h["flags"] == 3
        assert h["n_params"] == sum(t[1].size for t in ts)
        for name, arr, layout, scales in ts:
            info = f.info(name)
            assert info.ndim == arr.ndim and info.layout == layout
            assert info.quant == (1 if scales is not None else 0)
            np.testing.assert_array_equal(f.array(name), arr)
            if scales is not None:
                np.testing.assert_array_equal(f.scales(name), scales)
            else:
                assert f.scales(name) is None
            assert info.crc == zlib.crc32(arr.tobytes())
            assert f.verify(name)


@needs_ref
def test_reference_loader_reads_the_same(repo_tmp):
    """The reference's own loader, on the same file, sees every tensor as
    ovb_ovw1_* does: dtype, rank, layout, quantisation, dims, size, scale
    count, and stored and recomputed CRC."""
    ts = sample_tensors(np.random.default_rng(6))
    p = str(repo_tmp / "m.ovw")
    ovw1.write(p, ts)
    with ovw1.OVW1File(p) as f:
        for name, arr, layout, scales in ts:
            ref, err = O.ref_ovw1_tensor(p, name)
            assert err is None, err
            t = f.info(name)
            assert (t.dtype, t.ndim, t.layout, t.quant) == \
                (ref["dtype"], ref["ndim"], ref["layout"], ref["quant"])
            assert [t.dims[k] for k in range(4)] == ref["dims"]
            assert t.nbytes == ref["nbytes"] and t.n_scales == ref["n_scales"]
            assert t.crc == ref["crc"] == ref["crc_computed"]


def test_reference_minimal_file(repo_tmp):
    """The 272-byte file of the reference's own loader test: one 2x2 fp32
    tensor "x" = 1, 2, 3, 4 (header 128 B, descriptor at 128, name at 192,
    payload at 256)."""
    b = bytearray(272)
    struct.pack_into("<8sIIIIQQQQQQ", b, 0, b"OMNIVOIC", 1, 0, 1, 128, 128, 192, 256, 272, 0, 4)
    struct.pack_into("<IIBBBB4IIQQQQ", b, 128, 0, 1, 0, 2, 0, 0, 2, 2, 0, 0, 0, 0, 256, 16, 0)
    b[192] = ord("x")
    b[256:272] = np.array([1, 2, 3, 4], np.float32).tobytes()
    p = repo_tmp / "ref_min.bin"
    p.write_bytes(bytes(b))
    with ovw1.OVW1File(str(p)) as f:
        t = f.info("x")
        assert t.ndim == 2 and t.dims[0] == 2 and t.dims[1] == 2 and t.nbytes == 16
        np.testing.assert_array_equal(f.array("x"), [[1, 2], [3, 4]])


def _file(repo_tmp, rng):
    p = str(repo_tmp / "base.ovw")
    ovw1.write(p, sample_tensors(rng))
    return bytearray(open(p, "rb").read())


def _desc_off(b, i):
    index_off = struct.unpack_from("<Q", b, 24)[0]
    return index_off + 64 * i


@pytest.mark.parametrize("case,msg", [
    ("magic", "bad magic"), ("version", "unsupported version 2"), ("size", "file size mismatch"),
    ("index", "index out of bounds"), ("name", "tensor name out of bounds"),
    ("payload", "tensor payload out of bounds"), ("scales", "scales out of bounds"),
    ("nbytes", "size mismatch for 'layers.0.q_proj.weight'"), ("short", "smaller than a header"),
])
def test_rejects_like_the_reference(repo_tmp, case, msg):
    b = _file(repo_tmp, np.random.default_rng(2))
    d1 = _desc_off(b, 1)  # layers.0.q_proj.weight
    if case == "magic":
        b[0:8] = b"OMNIVOIX"
    elif case == "version":
        struct.pack_into("<I", b, 8, 2)
    elif case == "size":
        b += b"\0" * 64
    elif case == "index":
        struct.pack_into("<I", b, 16, 10_000)
    elif case == "name":
        struct.pack_into("<I", b, d1 + 4, len(b))
    elif case == "payload":
        struct.pack_into("<Q", b, d1 + 40, len(b) - 8)
    elif case == "scales":
        struct.pack_into("<Q", b, d1 + 56, len(b) - 16)
    elif case == "nbytes":
        struct.pack_into("<Q", b, d1 + 48, 96 * 64 - 1)
    elif case == "short":
        b = b[:40]
    p = repo_tmp / "bad.ovw"
    p.write_bytes(bytes(b))
    with pytest.raises(ValueError, match=msg) as e:
        ovw1.OVW1File(str(p))
    if O.ref_available():  # the reference's loader rejects it with the same message
        _, ref_err = O.ref_ovw1_tensor(str(p), "layers.0.q_proj.weight")
        assert ref_err is not None and ref_err == str(e.value)


def test_rejects_wrapping_scale_offset(repo_tmp):
    """A scales offset so large that offset + bytes wraps past 2^64 is out of
    bounds (not compared with the reference loader, whose check is a plain
    sum)."""
    b = _file(repo_tmp, np.random.default_rng(2))
    d1 = _desc_off(b, 1)
    struct.pack_into("<Q", b, d1 + 56, (1 << 64) - 8)
    p = repo_tmp / "wrap.ovw"
    p.write_bytes(bytes(b))
    with pytest.raises(ValueError, match="scales out of bounds"):
        ovw1.OVW1File(str(p))


def test_missing_file_and_tensor(repo_tmp):
    with pytest.raises(ValueError, match="cannot open"):
        ovw1.OVW1File(str(repo_tmp / "nope.ovw"))
    p = str(repo_tmp / "m.ovw")
    ovw1.write(p, sample_tensors(np.random.default_rng(3)))
    with ovw1.OVW1File(p) as f:
        with pytest.raises(ValueError, match="tensor not found: 'absent'"):
            f.info("absent")
        with pytest.raises(ValueError, match="out of range"):
            f.info(99)


def test_crc_detects_corruption(repo_tmp):
    rng = np.random.default_rng(4)
    ts = [("a%d" % n, rng.integers(-127, 128, size=n, dtype=np.int8), 0, None)
          for n in (1, 7, 8, 9, 63, 64, 65, 1000, 4099)]
    p = str(repo_tmp / "c.ovw")
    ovw1.write(p, ts)
    b = bytearray(open(p, "rb").read())
    with ovw1.OVW1File(p) as f:
        assert all(f.verify(t[0]) for t in ts)
    i = [t[0] for t in ts].index("a1000")
    off = struct.unpack_from("<Q", b, _desc_off(b, i) + 40)[0]
    b[off + 500] ^= 0x10
    q = repo_tmp / "c2.ovw"
    q.write_bytes(bytes(b))
    with ovw1.OVW1File(str(q)) as f:
        assert not f.verify("a1000")
        assert all(f.verify(t[0]) for t in ts if t[0] != "a1000")


@pytest.mark.parametrize("name,msg", [("model.norm.weight", "expected a 2-D weight"),
                                      ("conv.weight", "expected a 2-D weight"),
                                      ("absent", "tensor not found")])
def test_weight_rejects_non_int8_linear(repo_tmp, name, msg):
    """Rejected before any device call, so this runs without a GPU."""
    import ctypes as C

    from ovnative_b200 import _lib as L
    p = str(repo_tmp / "m.ovw")
    ts = sample_tensors(np.random.default_rng(5))
    ts.append(("fp32_linear", np.zeros((8, 4), np.float32), 1, None))
    ovw1.write(p, ts)
    with ovw1.OVW1File(p) as f:
        out = C.c_void_p()
        for nm, m in ((name, msg), ("fp32_linear", "not an int8 weight")):
            assert L.lib().ovb_ovw1_weight(f._h, nm.encode(), 0, None, C.byref(out)) == \
                L.OVB_ERR_INVALID_ARG
            assert m in L.lib().ovb_last_error().decode()
