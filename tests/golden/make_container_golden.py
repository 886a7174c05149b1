"""Generate `.tsk` container fixtures with the tensorshrink reference's own
writer (container.py), for the container reader's parity tests.

    python tests/golden/make_container_golden.py /path/to/tensorshrink

The reference container imports the `zstandard` package, which this
environment does not have; a stand-in module exposing the two calls the
reference makes (`ZstdCompressor(level=, threads=).compress(bytes)` and
`ZstdDecompressor().decompress(bytes)`) is registered first, backed by the
system libzstd through `tensorshrink_b200.zstd`. It writes and reads plain
single zstd frames, which is what `zstandard` produces for these calls.

Outputs (small files, committed):
* `tests/golden/ref_container.tsk` -- written by the reference
  `ContainerWriter` (quantized entries: uniform 4-bit with padding, NF4 with
  double quantization, 2-bit Lloyd-Max, 8-bit; raw entries: bf16 and fp32);
* `tests/golden/ref_container.npz` -- what the reference `ContainerReader`
  returns for each entry (`get_quantized` arrays, `get` of the raw ones).
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
HERE = Path(__file__).resolve().parent


def _zstd_standin():
    from tensorshrink_b200 import zstd as z
    m = types.ModuleType("zstandard")

    class ZstdCompressor:
        def __init__(self, level=3, threads=0, **_):
            self.level = level

        def compress(self, data):
            return z.compress(data, self.level)

    class ZstdDecompressor:
        def decompress(self, data):
            return z.decompress(data)

    m.ZstdCompressor, m.ZstdDecompressor = ZstdCompressor, ZstdDecompressor
    sys.modules["zstandard"] = m


def load_reference(path: str):
    _zstd_standin()
    pkg = types.ModuleType("tensorshrink")
    pkg.__path__ = [path]
    sys.modules["tensorshrink"] = pkg
    import importlib
    return importlib.import_module("tensorshrink.codec"), importlib.import_module("tensorshrink.container")


def student_t(shape, seed):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(shape, generator=g)
    chi = torch.randn((4,) + tuple(shape), generator=g).pow(2).sum(0)
    w = z / torch.sqrt(chi / 4.0)
    return (w * (0.02 / w.std())).to(torch.float16)


def main(ref_path: str) -> None:
    codec, container = load_reference(ref_path)
    torch.manual_seed(0)
    entries = {
        "layers.0.u4_pad.weight": (student_t((200, 300), 1), dict(bits=4, group_size=128, outlier_frac=0.003)),
        "layers.1.nf4_dq.weight": (student_t((256, 512), 2),
                                   dict(bits=4, group_size=128, outlier_frac=0.001, double_quant=True,
                                        nf_quant=True)),
        "layers.2.lloyd2.weight": (student_t((128, 256), 3),
                                   dict(bits=2, group_size=64, outlier_frac=0.002, companded=True)),
        "layers.3.u8.weight": (student_t((96, 640), 4), dict(bits=8, group_size=128, outlier_frac=0.001)),
    }
    raws = {"layers.0.bias": torch.randn(200).to(torch.bfloat16), "norm.weight": torch.rand(300)}
    out = {}
    path = HERE / "ref_container.tsk"
    with container.ContainerWriter(path) as wr:
        for name, (w, kw) in entries.items():
            qt = codec.quantize_tensor(w, **kw)
            wr.add_quantized(name, qt, rel_error=float(codec.relative_error(w, qt)))
        for name, t in raws.items():
            wr.add_raw(name, t)
    rd = container.ContainerReader(path)
    for name in entries:
        qt = rd.get_quantized(name)
        for f in ("packed", "scale", "gmin", "outlier_idx", "outlier_val", "codebook"):
            v = getattr(qt, f, None)
            if v is not None:
                out[f"{name}/{f}"] = np.asarray(v)
        out[f"{name}/meta"] = np.array([qt.bits, qt.group_size, qt.rows, qt.cols, qt.padded_cols, qt.n_groups])
    for name in raws:
        out[f"{name}/value"] = rd.get(name).float().numpy()
    rd.close()
    np.savez_compressed(HERE / "ref_container.npz", **out)
    print("wrote", path, path.stat().st_size, "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_container_golden.py /path/to/tensorshrink")
    main(sys.argv[1])
