"""Generate the golden parity fixtures by running the tensorshrink reference.

Run from the repository root, in a container where the reference checkout
is mounted (pass its path as the first argument):

    python tests/golden/make_golden.py /path/to/tensorshrink

The reference is imported without executing its package `__init__` (which
needs zstandard for the container module): a namespace package named
`tensorshrink` is pointed at the checkout and `codec`, `modules` are loaded
from it. Every case below runs the reference's own CPU path on seeded
synthetic weights and stores inputs and outputs in `golden.npz`:

* `codec.quantize_tensor` outputs (packed, scale, gmin, dq codes/meta,
  outlier idx/val, codebook);
* the `QuantLinear` buffers built from them (outlier row/col/delta);
* `y_ref = x @ dequantize_tensor(qt).T (+bias)` in fp32 and the CPU
  `QuantLinear.forward` output in the activation dtype;
* NF codebooks and double-quant round trips.

The fixtures are the only place the reference's behaviour enters the tests;
nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "golden.npz"


def load_reference(path: str):
    pkg = types.ModuleType("tensorshrink")
    pkg.__path__ = [path]
    sys.modules["tensorshrink"] = pkg
    import importlib
    codec = importlib.import_module("tensorshrink.codec")
    modules = importlib.import_module("tensorshrink.modules")
    return codec, modules


def student_t(shape, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    # Student-t(df=4) = N(0,1) / sqrt(chi2_4 / 4), drawn from one seeded generator.
    z = torch.randn(shape, generator=g)
    chi = torch.randn((4,) + tuple(shape), generator=g).pow(2).sum(0)
    w = z / torch.sqrt(chi / 4.0)
    w = w * (0.02 / w.std())
    return w.to(dtype)


CASES = [
    # name, shape, dtype, bits, gs, frac, dq, mode, bias, M, xdtype
    ("nf4_dq_g128", (96, 384), torch.float16, 4, 128, 0.001, True, "nf", False, 3, torch.float16),
    ("u4_g128_pad", (80, 300), torch.float16, 4, 128, 0.003, False, "uniform", True, 2, torch.float16),
    ("lloyd2_g64", (64, 512), torch.float16, 2, 64, 0.001, False, "lloyd", False, 4, torch.bfloat16),
    ("u8_dq_g128", (48, 256), torch.float16, 8, 128, 0.001, True, "uniform", True, 1, torch.float16),
    ("u2_g128_pad", (40, 250), torch.float16, 2, 128, 0.002, False, "uniform", False, 2, torch.float16),
    ("nf4_dq_g64", (64, 256), torch.float16, 4, 64, 0.001, True, "nf", False, 2, torch.bfloat16),
    ("u4_ties", (32, 256), torch.float16, 4, 128, 0.01, False, "uniform", False, 1, torch.float16),
    ("u4_dq_noout", (64, 256), torch.float16, 4, 128, 0.0, True, "uniform", False, 1, torch.float16),
    ("nf4_dq_pad_super", (50, 384), torch.float16, 4, 128, 0.001, True, "nf", True, 5, torch.float16),
    ("nf4_dq_bf16w", (64, 384), torch.bfloat16, 4, 128, 0.001, True, "nf", False, 2, torch.bfloat16),
    ("u4_f32w", (48, 256), torch.float32, 4, 128, 0.002, False, "uniform", False, 2, torch.float16),
    ("nf8_g128", (32, 256), torch.float16, 8, 128, 0.001, False, "nf", False, 1, torch.float16),
    ("nf2_dq_g64", (48, 320), torch.float16, 2, 64, 0.001, True, "nf", False, 2, torch.float16),
    ("lloyd4_g128", (64, 384), torch.float16, 4, 128, 0.001, False, "lloyd", False, 2, torch.float16),
    ("nf4_dq_big", (512, 1024), torch.float16, 4, 128, 0.001, True, "nf", False, 1, torch.float16),
    ("lloyd2_sampled", (600, 640), torch.float16, 2, 64, 0.001, False, "lloyd", False, 2, torch.bfloat16),
]


def main(ref_path: str) -> None:
    codec, modules = load_reference(ref_path)
    # Record the float32 Lloyd-Max levels the reference assigns codes against
    # (it stores only their fp16 rounding in QuantizedTensor.codebook).
    fitted = []
    real_fit = codec._fit_lloyd_max_1d

    def recording_fit(*a, **kw):
        cent = real_fit(*a, **kw)
        fitted.append(cent.clone())
        return cent

    codec._fit_lloyd_max_1d = recording_fit
    out = {}
    names = []
    for ci, (name, shape, wdt, bits, gs, frac, dq, mode, has_bias, M, xdt) in enumerate(CASES):
        torch.manual_seed(1000 + ci)
        w = student_t(shape, 7 + ci, wdt)
        if name == "u4_ties":
            # few distinct magnitudes -> many elements tie at the top-k threshold
            w = (torch.round(w.float() / 0.01) * 0.01).to(wdt)
        torch.manual_seed(2000 + ci)   # Lloyd-Max sampling draws from the global RNG
        fitted.clear()
        qt = codec.quantize_tensor(w, bits=bits, group_size=gs, outlier_frac=frac,
                                   double_quant=dq, companded=(mode == "lloyd"),
                                   nf_quant=(mode == "nf"))
        g = torch.Generator().manual_seed(3000 + ci)
        x = torch.randn((M, shape[1]), generator=g).to(xdt)
        bias = (torch.randn(shape[0], generator=g) * 0.1).to(xdt) if has_bias else None
        W = codec.dequantize_tensor(qt, dtype=torch.float32)
        y_ref = x.float() @ W.T
        if bias is not None:
            y_ref = y_ref + bias.float()
        ql = modules.QuantLinear(qt, bias, use_triton=False)
        y_cpu = ql(x)
        p = f"{name}/"
        names.append(name)
        out[p + "w"] = w.float().numpy() if wdt == torch.bfloat16 else w.numpy()
        out[p + "w_dtype"] = np.array(str(wdt).replace("torch.", ""))
        out[p + "params"] = np.array([bits, gs, int(dq), M], dtype=np.int64)
        out[p + "frac"] = np.array(frac, dtype=np.float64)
        out[p + "mode"] = np.array(mode)
        for f in ("packed", "scale", "gmin", "outlier_idx", "outlier_val", "dq_scale_codes",
                  "dq_scale_meta", "dq_gmin_codes", "dq_gmin_meta", "codebook"):
            v = getattr(qt, f)
            if v is not None:
                out[p + f] = v
        if fitted:
            out[p + "lloyd_cb32"] = fitted[-1].numpy()
        out[p + "ql_outlier_row"] = ql.outlier_row.numpy()
        out[p + "ql_outlier_col"] = ql.outlier_col.numpy()
        out[p + "ql_outlier_delta"] = ql.outlier_delta.numpy()
        out[p + "x"] = x.float().numpy()
        out[p + "x_dtype"] = np.array(str(xdt).replace("torch.", ""))
        if bias is not None:
            out[p + "bias"] = bias.float().numpy()
        out[p + "y_ref"] = y_ref.numpy()
        out[p + "y_cpu"] = y_cpu.float().numpy()
        print(f"{name:18s} k={qt.outlier_idx.shape[0]:6d} packed={qt.packed.shape}")
    out["cases"] = np.array(names)
    for bits in (2, 4, 8):
        out[f"nf_codebook/{bits}"] = codec._get_nf_codebook(bits)
    # double-quant round trip on a ragged length (pads the last super-group)
    g = torch.Generator().manual_seed(77)
    vals = (torch.rand(1000, generator=g) * 0.01).to(torch.float16).numpy()
    c, m = codec._double_quantize_np(vals, 256)
    out["dq/vals"], out["dq/codes"], out["dq/meta"] = vals, c, m
    out["dq/recon16"] = codec._double_dequantize_np(c, m, vals.shape)
    # Lloyd fit on a fixed sample (deterministic: no sampling below the cap)
    torch.manual_seed(5)
    sample = torch.randn(5000) * 3 + 7
    out["lloyd/sample"] = sample.numpy()
    for lv in (4, 16):
        out[f"lloyd/cent{lv}"] = real_fit(sample, lv).numpy()
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py /path/to/tensorshrink")
    main(sys.argv[1])
