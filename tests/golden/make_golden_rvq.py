"""Generate fixtures for smooth-scaled and 6-bit RVQ quantization by running
the tensorshrink reference's own codec (codec.py:519-525 smoothing,
678-737 `_quantize_rvq`, 810-847 `_dequantize_rvq`):

    python tests/golden/make_golden_rvq.py /path/to/tensorshrink

Writes tests/golden/golden_rvq.npz: per case the input weight, every
QuantizedTensor field the reference fills (including smooth_scale and the
stage-2 arrays) and `dequantize_tensor`'s fp32 reconstruction.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from make_golden import load_reference, student_t  # noqa: E402

CASES = [
    # name, shape, bits, gs, frac, dq, smooth, alpha, nf
    ("smooth_u4", (96, 384), 4, 128, 0.002, False, True, 0.5, False),
    ("smooth_nf4_dq", (64, 512), 4, 128, 0.001, True, True, 0.3, True),
    ("rvq6", (80, 300), 6, 128, 0.003, False, False, 0.5, False),
    ("rvq6_dq_smooth", (64, 512), 6, 64, 0.001, True, True, 0.5, False),
]


def main(ref_path: str) -> None:
    codec, _ = load_reference(ref_path)
    out, names = {}, []
    for ci, (name, shape, bits, gs, frac, dq, smooth, alpha, nf) in enumerate(CASES):
        w = student_t(shape, 50 + ci, torch.float16)
        qt = codec.quantize_tensor(w, bits=bits, group_size=gs, outlier_frac=frac, double_quant=dq,
                                   smooth=smooth, smooth_alpha=alpha, nf_quant=nf)
        p = f"{name}/"
        names.append(name)
        out[p + "w"] = w.numpy()
        out[p + "params"] = np.array([bits, gs, int(dq), int(smooth), int(nf)], dtype=np.int64)
        out[p + "frac"] = np.array(frac)
        out[p + "alpha"] = np.array(alpha)
        for f in ("packed", "scale", "gmin", "outlier_idx", "outlier_val", "dq_scale_codes", "dq_scale_meta",
                  "dq_gmin_codes", "dq_gmin_meta", "codebook", "smooth_scale", "stage2_packed",
                  "stage2_scale", "stage2_gmin"):
            v = getattr(qt, f, None)
            if v is not None:
                out[p + f] = v
        out[p + "W"] = codec.dequantize_tensor(qt, dtype=torch.float32).numpy()
        print(f"{name:16s} bits={qt.bits} k={qt.outlier_idx.shape[0]}")
    out["cases"] = np.array(names)
    np.savez_compressed(HERE / "golden_rvq.npz", **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden_rvq.py /path/to/tensorshrink")
    main(sys.argv[1])
