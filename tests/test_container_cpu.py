"""The `.tsk` container against files written by the reference's own
ContainerWriter (tests/golden/ref_container.tsk, made by
tests/golden/make_container_golden.py), on the host.

* every entry read back equals what the reference ContainerReader returned;
* rewriting the reference's tensors with this writer gives the same
  decompressed blobs and part tables byte for byte (so the reference reader
  reads our files);
* round trips, the double-quant extension and the CPU QuantLinear built
  from an entry.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from tensorshrink_b200 import container as ct
from tensorshrink_b200 import zstd
from tensorshrink_b200.modules import QuantLinear

GOLD = Path(__file__).resolve().parent / "golden"
TSK = GOLD / "ref_container.tsk"


@pytest.fixture(scope="module")
def ref():
    with np.load(GOLD / "ref_container.npz") as z:
        return {k: z[k] for k in z.files}


def test_reads_reference_container(ref):
    with ct.ContainerReader(TSK) as rd:
        assert rd.stats()["n_quantized"] == 4 and rd.stats()["n_raw"] == 2
        for name in rd.names():
            if rd.kind(name) == "raw":
                np.testing.assert_array_equal(rd.get(name).float().numpy(), ref[f"{name}/value"])
                continue
            qt = rd.get_quantized(name)
            meta = ref[f"{name}/meta"]
            assert [qt.bits, qt.group_size, qt.rows, qt.cols, qt.padded_cols, qt.n_groups] == list(meta)
            for f in ("packed", "scale", "gmin", "outlier_idx", "outlier_val", "codebook"):
                key = f"{name}/{f}"
                if key in ref:
                    np.testing.assert_array_equal(getattr(qt, f), ref[key], err_msg=key)
        assert rd.get("layers.0.bias").dtype == torch.bfloat16


def test_writer_blobs_match_reference(tmp_path):
    """Same tensors through this writer: identical decompressed blobs and
    part tables, the same manifest fields."""
    out = tmp_path / "ours.tsk"
    with ct.ContainerReader(TSK) as rd, ct.ContainerWriter(out) as wr:
        for name in rd.names():
            e = rd.entry(name)
            if e["kind"] == "raw":
                wr.add_raw(name, rd.get(name))
            else:
                wr.add_quantized(name, rd.get_quantized(name), rel_error=e["rel_error"],
                                 escalated=e["escalated"])
    with ct.ContainerReader(TSK) as a, ct.ContainerReader(out) as b:
        assert a.names() == b.names()
        for name in a.names():
            ea, eb = a.entry(name), b.entry(name)
            skip = {"segments_v2", "segments"}
            assert {k: v for k, v in ea.items() if k not in skip} == {k: v for k, v in eb.items() if k not in skip}
            if ea["kind"] == "quant":
                ra, pa = a._blob(ea)
                rb, pb = b._blob(eb)
                assert pa == pb and ra == rb, name
            else:
                sa, sb = ea["segments"]["data"], eb["segments"]["data"]
                assert (sa["np_dtype"], sa["shape"]) == (sb["np_dtype"], sb["shape"])
                assert zstd.decompress(a._frame(sa["offset"], sa["length"])) == \
                    zstd.decompress(b._frame(sb["offset"], sb["length"]))


def test_outlier_stream_codec():
    rng = np.random.default_rng(0)
    for cols in (300, 70000):                 # 16-bit, then 32-bit indices
        idx = np.sort(rng.choice(50 * cols, size=400, replace=False)).astype(np.int32)
        val = rng.standard_normal(400).astype(np.float16)
        rd, c, v, dt = ct.encode_outliers(idx, val, cols)
        assert dt == ("uint16" if cols < 65536 else "uint32")
        np.testing.assert_array_equal(ct.decode_outliers(rd, c, cols), idx)
        np.testing.assert_array_equal(v, val)
    e = ct.encode_outliers(np.zeros(0, np.int32), np.zeros(0, np.float16), 10)
    assert e[0].size == 0 and ct.decode_outliers(e[0], e[1], 10).size == 0


def test_double_quant_extension_round_trip(tmp_path):
    """Double-quantized weights keep their compact metadata (extra parts)."""
    from tests.test_host_cpu import qt_from_case
    from tests.conftest import load_case, GOLDEN
    with np.load(GOLDEN) as z:
        g = {k: z[k] for k in z.files}
    qt = qt_from_case(load_case(g, "nf4_dq_g128"))
    p = tmp_path / "dq.tsk"
    with ct.ContainerWriter(p) as wr:
        wr.add_quantized("w", qt)
    with ct.ContainerReader(p) as rd:
        assert rd.entry("w")["double_quant"] and rd.entry("w")["dq_group_size"] == 256
        back = rd.get_quantized("w")
    for f in ("packed", "scale", "gmin", "dq_scale_codes", "dq_scale_meta", "dq_gmin_codes", "dq_gmin_meta",
              "codebook"):
        np.testing.assert_array_equal(getattr(back, f), getattr(qt, f), err_msg=f)
    order = np.argsort(qt.outlier_idx, kind="stable")
    np.testing.assert_array_equal(np.sort(back.outlier_idx), qt.outlier_idx[order])


def test_cpu_quantlinear_from_container():
    with ct.ContainerReader(TSK) as rd:
        for name in ("layers.0.u4_pad.weight", "layers.2.lloyd2.weight"):
            qt = rd.get_quantized(name)
            a = QuantLinear(qt)
            b = rd.to_quantlinear(name, "cpu")
            x = torch.randn(3, qt.cols)
            torch.testing.assert_close(a(x), b(x), rtol=0, atol=0)


def test_bad_magic(tmp_path):
    p = tmp_path / "x.tsk"
    p.write_bytes(b"0" * 64)
    with pytest.raises(ValueError, match="magic"):
        ct.ContainerReader(p)
