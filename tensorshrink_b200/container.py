"""The `.tsk` container: a whole quantized state_dict in one file, read
straight into QuantLinear device buffers.

Same on-disk format as the reference (container.py:1-460), so files move
between the two libraries in both directions:

    [zstd segment of tensor 1] ... [zstd segment of tensor N]
    [manifest JSON, utf-8] [u64 LE manifest length] [b"TSHRNK01"]

A quantized entry (manifest "segments_v2") is one zstd frame holding its
arrays back to back ("parts": offset/length/dtype/shape inside the
decompressed blob): packed, scale, gmin, outlier_row_delta, outlier_col,
outlier_val (outliers row-sorted, rows stored as deltas, "outlier_encoding":
"delta_row_v1"), and codebook when companded. Older "segments" entries (one
frame per array, flat outlier_idx) are read too. A raw entry holds one
tensor (bf16 widened to fp32 on disk, cast back on read).

Extension, written by this library only: double-quantized weights also
store their compact metadata as parts dq_scale_codes, dq_scale_meta,
dq_gmin_codes, dq_gmin_meta ("double_quant": true, "dq_group_size"). The
fp16 scale/gmin parts are still written (reconstructed), so the reference
reader loads such files unchanged; it ignores the extra parts.

Loading to the GPU (`ContainerReader.to_quantlinear`): the frame is
decompressed on the host (libzstd, threads for several entries), the parts
are copied to the device, and `ts_outlier_tables_from_stream` turns the
outlier stream into QuantLinear's row/col/delta/CSR tables on the device.
"""

from __future__ import annotations

import ctypes as C
import io
import json
import mmap
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from types import SimpleNamespace
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np
import torch

from . import zstd
from .codec import DeviceQuant, QuantizedTensor

MAGIC = b"TSHRNK01"
ZSTD_LEVEL = 12
ZSTD_LEVEL_MAX = 19
CONTAINER_FORMAT_VERSION = 2


# ---------------------------------------------------------------------------
# outlier stream (container.py:98-153)
# ---------------------------------------------------------------------------

def encode_outliers(outlier_idx: np.ndarray, outlier_val: np.ndarray, cols: int):
    """Flat outlier indices -> (row deltas, columns, values, dtype name),
    stably sorted by row; 16-bit indices when every delta and column fits,
    else 32-bit."""
    n = int(outlier_idx.shape[0])
    if n == 0:
        z = np.zeros(0, dtype=np.uint16)
        return z, z.copy(), np.asarray(outlier_val), "uint16"
    flat = outlier_idx.astype(np.int64)
    order = np.argsort(flat // cols, kind="stable")
    rows, cols_ = (flat // cols)[order], (flat % cols)[order]
    deltas = np.diff(rows, prepend=0)
    small = deltas.max() < 65536 and cols - 1 < 65536
    dt = np.uint16 if small else np.uint32
    return deltas.astype(dt), cols_.astype(dt), np.asarray(outlier_val)[order], np.dtype(dt).name


def decode_outliers(row_delta: np.ndarray, col: np.ndarray, cols: int) -> np.ndarray:
    """(row deltas, columns) -> flat int32 indices row * cols + col."""
    if row_delta.shape[0] == 0:
        return np.zeros(0, dtype=np.int32)
    rows = np.cumsum(row_delta.astype(np.int64))
    return (rows * cols + col.astype(np.int64)).astype(np.int32)


# ---------------------------------------------------------------------------
# writer
# ---------------------------------------------------------------------------

def _as_qt(obj) -> QuantizedTensor:
    """QuantizedTensor from a QuantizedTensor, DeviceQuant or QuantLinear."""
    if isinstance(obj, QuantizedTensor):
        return obj
    if hasattr(obj, "to_quantized_tensor"):
        return obj.to_quantized_tensor()
    raise TypeError(f"cannot store {type(obj).__name__} as a quantized entry")


def quantized_entry(qt: QuantizedTensor, rel_error: Optional[float] = None, escalated: Optional[bool] = None,
                    force_fp32_compute: bool = False) -> Tuple[dict, bytes]:
    """Manifest entry (without file offsets) and the uncompressed blob of one
    quantized tensor (container.py:156-218)."""
    if qt.bits == 6 or qt.stage2_packed is not None:
        raise NotImplementedError("6-bit RVQ tensors are not stored by this container writer")
    entry = {
        "kind": "quant", "orig_shape": list(qt.orig_shape), "orig_dtype": qt.orig_dtype, "bits": qt.bits,
        "group_size": qt.group_size, "rows": qt.rows, "cols": qt.cols, "padded_cols": qt.padded_cols,
        "n_groups": qt.n_groups, "n_outliers": qt.n_outliers(), "rel_error": rel_error,
        "escalated": bool(escalated) if escalated is not None else None,
        "force_fp32_compute": bool(force_fp32_compute), "outlier_encoding": "delta_row_v1",
    }
    row_delta, col, val, _ = encode_outliers(qt.outlier_idx, qt.outlier_val, qt.cols)
    arrays = [("packed", qt.packed), ("scale", qt.scale), ("gmin", qt.gmin), ("outlier_row_delta", row_delta),
              ("outlier_col", col), ("outlier_val", val)]
    if qt.codebook is not None:
        arrays.append(("codebook", qt.codebook))
        entry["companded"] = True
    if qt.dq_scale_codes is not None:
        arrays += [("dq_scale_codes", qt.dq_scale_codes), ("dq_scale_meta", qt.dq_scale_meta),
                   ("dq_gmin_codes", qt.dq_gmin_codes), ("dq_gmin_meta", qt.dq_gmin_meta)]
        entry["double_quant"] = True
        entry["dq_group_size"] = int(qt.dq_scale_codes.shape[0] // qt.dq_scale_meta.shape[0])
    parts, chunks, off = {}, [], 0
    for name, arr in arrays:
        a = np.ascontiguousarray(arr)
        parts[name] = {"offset": off, "length": a.nbytes, "np_dtype": str(a.dtype), "shape": list(a.shape)}
        chunks.append(a.tobytes())
        off += a.nbytes
    entry["_parts"] = parts
    return entry, b"".join(chunks)


def raw_entry(tensor: torch.Tensor) -> Tuple[dict, bytes]:
    """Manifest entry and blob of a tensor stored as is (container.py:221-240)."""
    t = tensor.detach().to("cpu").contiguous()
    dtype_name = str(t.dtype).replace("torch.", "")
    if t.dtype == torch.bfloat16:
        t = t.to(torch.float32)   # numpy has no bf16; the widening is exact
    a = t.numpy()
    return ({"kind": "raw", "orig_shape": list(tensor.shape), "orig_torch_dtype": dtype_name,
             "np_dtype": str(a.dtype), "_data_shape": list(a.shape)}, a.tobytes())


class ContainerWriter:
    """Append-only writer (container.py:243-330): each tensor's frame is
    written as it is added; the manifest and footer on close()."""

    def __init__(self, path):
        self.path = str(path)
        self._f = open(self.path, "wb")
        self._manifest = {"format": "tensorshrink-v1", "format_version": CONTAINER_FORMAT_VERSION, "tensors": {}}
        self._offset = 0

    def add_precompressed(self, name: str, entry: dict, frame: bytes) -> None:
        off, ln = self._offset, len(frame)
        self._f.write(frame)
        self._offset += ln
        entry = dict(entry)
        if entry["kind"] == "quant":
            entry["segments_v2"] = {"blob": {"offset": off, "length": ln}, "parts": entry.pop("_parts")}
        else:
            shape = entry.pop("_data_shape")
            entry["segments"] = {"data": {"offset": off, "length": ln, "np_dtype": entry["np_dtype"],
                                          "shape": shape}}
        self._manifest["tensors"][name] = entry

    def add_quantized(self, name: str, qt, rel_error: Optional[float] = None, escalated: Optional[bool] = None,
                      force_fp32_compute: bool = False, level: int = ZSTD_LEVEL) -> None:
        entry, blob = quantized_entry(_as_qt(qt), rel_error, escalated, force_fp32_compute)
        self.add_precompressed(name, entry, zstd.compress(blob, level))

    def add_raw(self, name: str, tensor: torch.Tensor, level: int = ZSTD_LEVEL) -> None:
        entry, blob = raw_entry(tensor)
        self.add_precompressed(name, entry, zstd.compress(blob, level))

    def close(self) -> None:
        if self._f.closed:
            return
        m = json.dumps(self._manifest).encode("utf-8")
        self._f.write(m)
        self._f.write(struct.pack("<Q", len(m)))
        self._f.write(MAGIC)
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        if exc_type is None:
            self.close()
        else:
            self._f.close()


# ---------------------------------------------------------------------------
# reader
# ---------------------------------------------------------------------------

_TORCH_OF_NP = {"uint8": torch.uint8, "uint16": torch.int16, "int16": torch.int16, "uint32": torch.int32,
                "int32": torch.int32, "float16": torch.float16, "float32": torch.float32, "int64": torch.int64}


class ContainerReader:
    """Reader (container.py:338-520): the manifest from the footer, then any
    entry by its offsets through a read-only mmap."""

    def __init__(self, path):
        self.path = str(path)
        self._f = open(self.path, "rb")
        self._f.seek(-len(MAGIC), io.SEEK_END)
        if self._f.read(len(MAGIC)) != MAGIC:
            raise ValueError(f"{path} is not a tensorshrink container (bad magic footer)")
        self._f.seek(-(len(MAGIC) + 8), io.SEEK_END)
        (mlen,) = struct.unpack("<Q", self._f.read(8))
        self._f.seek(-(len(MAGIC) + 8 + mlen), io.SEEK_END)
        self.manifest = json.loads(self._f.read(mlen))
        try:
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        except (ValueError, OSError):
            self._mm = None

    # -- catalogue ---------------------------------------------------------------------
    def names(self) -> List[str]:
        return list(self.manifest["tensors"].keys())

    def kind(self, name: str) -> str:
        return self.manifest["tensors"][name]["kind"]

    def entry(self, name: str) -> dict:
        return self.manifest["tensors"][name]

    def stats(self) -> dict:
        """Per-kind counts and byte totals (container.py:466-495)."""
        total = os.path.getsize(self.path)
        n_q = sum(1 for e in self.manifest["tensors"].values() if e["kind"] == "quant")
        return {"n_tensors": len(self.manifest["tensors"]), "n_quantized": n_q,
                "n_raw": len(self.manifest["tensors"]) - n_q, "file_bytes": total}

    # -- bytes -----------------------------------------------------------------------
    def _frame(self, offset: int, length: int) -> bytes:
        if self._mm is not None:
            return self._mm[offset: offset + length]
        self._f.seek(offset)
        return self._f.read(length)

    def _blob(self, entry: dict) -> Tuple[bytes, dict]:
        """Decompressed blob of a v2 quantized entry and its part table."""
        seg = entry["segments_v2"]
        return zstd.decompress(self._frame(seg["blob"]["offset"], seg["blob"]["length"])), seg["parts"]

    @staticmethod
    def _part(raw, parts: dict, name: str) -> np.ndarray:
        m = parts[name]
        dt = np.dtype(m["np_dtype"])
        return np.frombuffer(raw, dtype=dt, count=m["length"] // dt.itemsize, offset=m["offset"]).reshape(m["shape"])

    def _read_segment(self, seg: dict) -> np.ndarray:
        raw = zstd.decompress(self._frame(seg["offset"], seg["length"]))
        return np.frombuffer(raw, dtype=np.dtype(seg["np_dtype"])).reshape(seg["shape"]).copy()

    # -- host objects ---------------------------------------------------------------------
    def get_quantized(self, name: str) -> QuantizedTensor:
        """The entry as a host QuantizedTensor, still packed (container.py:424-431)."""
        e = self.entry(name)
        if e["kind"] != "quant":
            raise ValueError(f"tensor {name!r} is stored raw, not quantized")
        extra = {}
        if "segments_v2" in e:
            raw, parts = self._blob(e)
            p = lambda k: self._part(raw, parts, k).copy()  # noqa: E731
            packed, scale, gmin = p("packed"), p("scale"), p("gmin")
            codebook = p("codebook") if e.get("companded") else None
            if e.get("outlier_encoding") == "delta_row_v1":
                idx = decode_outliers(p("outlier_row_delta"), p("outlier_col"), e["cols"])
            else:
                idx = p("outlier_idx")
            val = p("outlier_val")
            if e.get("double_quant"):
                extra = {k: p(k) for k in ("dq_scale_codes", "dq_scale_meta", "dq_gmin_codes", "dq_gmin_meta")}
        else:
            s = e["segments"]
            packed, scale, gmin = (self._read_segment(s[k]) for k in ("packed", "scale", "gmin"))
            idx, val = self._read_segment(s["outlier_idx"]), self._read_segment(s["outlier_val"])
            codebook = None
        return QuantizedTensor(orig_shape=tuple(e["orig_shape"]), orig_dtype=e["orig_dtype"], bits=e["bits"],
                               group_size=e["group_size"], rows=e["rows"], cols=e["cols"],
                               padded_cols=e["padded_cols"], n_groups=e["n_groups"], packed=packed, scale=scale,
                               gmin=gmin, outlier_idx=idx, outlier_val=val, codebook=codebook, **extra)

    def get_quantized_many(self, names: Iterable[str], max_workers: Optional[int] = None
                           ) -> Dict[str, QuantizedTensor]:
        """Several entries, decompressed on a thread pool (libzstd runs without
        the GIL)."""
        names = list(names)
        if len(names) <= 1 or self._mm is None:
            return {n: self.get_quantized(n) for n in names}
        with ThreadPoolExecutor(max_workers=max_workers or min(32, 2 * (os.cpu_count() or 4))) as ex:
            return dict(zip(names, ex.map(self.get_quantized, names)))

    def get(self, name: str, device=None, dtype=None) -> torch.Tensor:
        """Raw entries as stored; quantized entries dequantized (exact outlier
        values) on the GPU (container.py:449-468)."""
        e = self.entry(name)
        if e["kind"] == "raw":
            t = torch.from_numpy(self._read_segment(e["segments"]["data"]))
            if e.get("orig_torch_dtype"):
                t = t.to(getattr(torch, e["orig_torch_dtype"]))
        else:
            from .codec import dequantize_tensor
            t = dequantize_tensor(self.get_quantized(name), device=device)
        if device is not None:
            t = t.to(device)
        if dtype is not None:
            t = t.to(dtype)
        return t

    # -- device ------------------------------------------------------------------------------
    def to_quantlinear(self, name: str, device="cuda", bias: Optional[torch.Tensor] = None,
                       force_fp32_compute: Optional[bool] = None):
        """Build a QuantLinear directly on `device` from a quantized entry:
        the decompressed parts are copied from pinned host memory, and the
        outlier stream becomes QuantLinear's row/col/delta/CSR tables on the
        device (`ts_outlier_tables_from_stream`). No host-side table build."""
        from . import _C, kernels
        from .modules import QuantLinear
        e = self.entry(name)
        if e["kind"] != "quant":
            raise ValueError(f"tensor {name!r} is stored raw, not quantized")
        dev = torch.device(device)
        if dev.type != "cuda":
            ql = QuantLinear(self.get_quantized(name), bias)
            return ql
        if "segments_v2" not in e or e.get("outlier_encoding") != "delta_row_v1":
            return QuantLinear(self.get_quantized(name), bias).to(dev)
        seg = e["segments_v2"]
        frame = self._frame(seg["blob"]["offset"], seg["blob"]["length"])
        host = torch.empty(zstd.decompressed_size(frame), dtype=torch.uint8, pin_memory=True)
        zstd.decompress_into(frame, host.numpy())
        parts = seg["parts"]

        def put(pname: str) -> torch.Tensor:
            m = parts[pname]
            t = torch.empty(m["length"], dtype=torch.uint8, device=dev)
            t.copy_(host[m["offset"]: m["offset"] + m["length"]], non_blocking=True)
            return t.view(_TORCH_OF_NP[m["np_dtype"]]).view(m["shape"]) if m["length"] else \
                torch.empty(m["shape"], dtype=_TORCH_OF_NP[m["np_dtype"]], device=dev)

        packed = put("packed")
        dq = bool(e.get("double_quant"))
        src = SimpleNamespace(
            orig_shape=tuple(e["orig_shape"]), orig_dtype=e["orig_dtype"], bits=e["bits"],
            group_size=e["group_size"], rows=e["rows"], cols=e["cols"], padded_cols=e["padded_cols"],
            n_groups=e["n_groups"], packed=packed, scale=put("scale"), gmin=put("gmin"),
            dq_scale_codes=put("dq_scale_codes") if dq else None, dq_scale_meta=put("dq_scale_meta") if dq else None,
            dq_gmin_codes=put("dq_gmin_codes") if dq else None, dq_gmin_meta=put("dq_gmin_meta") if dq else None,
            dq_group_size=int(e.get("dq_group_size", 0)) if dq else 0,
            codebook_store=put("codebook").to(torch.float32) if e.get("companded") else None)
        n = int(parts["outlier_val"]["shape"][0])
        ib = np.dtype(parts["outlier_col"]["np_dtype"]).itemsize
        rdelta, col, val = put("outlier_row_delta"), put("outlier_col"), put("outlier_val")
        src.outlier_row = torch.empty(n, dtype=torch.int32, device=dev)
        src.outlier_col = torch.empty(n, dtype=torch.int32, device=dev)
        src.outlier_delta = torch.empty(n, dtype=torch.float16, device=dev)
        src.outlier_row_ptr = torch.empty(e["rows"] + 1, dtype=torch.int32, device=dev)
        bad = torch.zeros(1, dtype=torch.int32, device=dev)
        qw = kernels.make_qweight(packed=packed, scale=src.scale, gmin=src.gmin, bits=src.bits,
                                  group_size=src.group_size, cols=src.cols, out_features=src.rows,
                                  n_groups=src.n_groups, codebook=src.codebook_store,
                                  dq_scale_codes=src.dq_scale_codes, dq_scale_meta=src.dq_scale_meta,
                                  dq_gmin_codes=src.dq_gmin_codes, dq_gmin_meta=src.dq_gmin_meta,
                                  dq_group_size=src.dq_group_size)
        with torch.cuda.device(dev):
            rc = _C.load().ts_outlier_tables_from_stream(
                qw, rdelta.data_ptr() if n else None, col.data_ptr() if n else None, ib,
                val.data_ptr() if n else None, n, src.outlier_row.data_ptr() if n else None,
                src.outlier_col.data_ptr() if n else None, src.outlier_delta.data_ptr() if n else None,
                src.outlier_row_ptr.data_ptr(), bad.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        _C.check(rc, "ts_outlier_tables_from_stream")
        if int(bad.item()):
            raise ValueError(f"{name!r}: outlier stream points outside the weight")
        fp32 = bool(e.get("force_fp32_compute", False)) if force_fp32_compute is None else force_fp32_compute
        if bias is not None:
            bias = bias.to(dev)
        return QuantLinear(None, bias, force_fp32_compute=fp32, _device_quant=src)

    def close(self) -> None:
        if self._mm is not None:
            self._mm.close()
            self._mm = None
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ---------------------------------------------------------------------------
# whole state_dicts and modules
# ---------------------------------------------------------------------------

def save_container(state_dict: Dict[str, torch.Tensor], out_path, **quantize_kwargs) -> dict:
    """Quantize every eligible tensor of a state_dict (on the GPU) and write
    the container (container.py:510-541): tensors of >= 2 dims and
    `min_numel` elements whose names match none of `skip_name_patterns` go
    through quantize_tensor_adaptive (allowed_bits 2/4/8 by default); the
    rest are stored raw."""
    from .codec import quantize_tensor_adaptive
    min_numel = quantize_kwargs.pop("min_numel", 16384)
    skip = quantize_kwargs.pop("skip_name_patterns",
                               ("norm", "bias", "position", "shared", "relative_attention_bias"))
    quantize_kwargs.setdefault("allowed_bits", (2, 4, 8))
    stats = {"tensors": [], "orig_bytes": 0}
    with ContainerWriter(out_path) as wr:
        for name, t in state_dict.items():
            nbytes = t.numel() * t.element_size()
            if t.dim() >= 2 and t.numel() >= min_numel and not any(p in name.lower() for p in skip):
                qt, err, esc = quantize_tensor_adaptive(t, **quantize_kwargs)
                wr.add_quantized(name, qt, rel_error=err, escalated=esc)
                stats["tensors"].append({"name": name, "bits": qt.bits, "rel_error": err, "orig_bytes": nbytes})
            else:
                wr.add_raw(name, t)
                stats["tensors"].append({"name": name, "bits": None, "rel_error": 0.0, "orig_bytes": nbytes})
            stats["orig_bytes"] += nbytes
    stats["file_bytes"] = os.path.getsize(str(out_path))
    return stats


def save_quant_module(model: torch.nn.Module, path, verbose: bool = True) -> dict:
    """Write a quantized model (modules.py:1458-1496): every QuantLinear as a
    quantized `<name>.weight` entry (its bias raw), every other state_dict
    entry outside the QuantLinear layers raw."""
    from .modules import QuantLinear
    done, prefixes = set(), []
    with ContainerWriter(path) as wr:
        for name, mod in model.named_modules():
            if isinstance(mod, QuantLinear):
                wr.add_quantized(f"{name}.weight", mod, force_fp32_compute=mod.force_fp32_compute)
                done.add(f"{name}.weight")
                prefixes.append(f"{name}.")
                if mod.bias is not None:
                    wr.add_raw(f"{name}.bias", mod.bias)
                    done.add(f"{name}.bias")
        n_raw = 0
        for key, t in model.state_dict().items():
            if key in done or any(key.startswith(p) for p in prefixes):
                continue
            wr.add_raw(key, t)
            n_raw += 1
    if verbose:
        print(f"  saved {len(done)} quantized-layer tensors + {n_raw} raw tensors -> {path}")
    return {"n_quant": len(done), "n_raw": n_raw}


def load_quantized_module(model: torch.nn.Module, reader: ContainerReader, device=None, verbose: bool = True,
                          **ignored) -> dict:
    """Fill a freshly built model from a container (modules.py:1499-1586):
    each nn.Linear whose `<name>.weight` is a quantized entry becomes a
    QuantLinear (built on `device` directly when it is a CUDA device), and
    the raw entries are loaded with load_state_dict(strict=False)."""
    from .modules import QuantLinear, _set_module_by_name
    names = set(reader.names())
    replaced = 0
    for name, mod in list(model.named_modules()):
        if isinstance(mod, torch.nn.Linear) and not isinstance(mod, QuantLinear):
            wkey, bkey = f"{name}.weight", f"{name}.bias"
            if wkey in names and reader.kind(wkey) == "quant":
                bias = reader.get(bkey) if bkey in names else None
                ql = reader.to_quantlinear(wkey, device or mod.weight.device, bias=bias)
                _set_module_by_name(model, name, ql)
                replaced += 1
    keys = set(model.state_dict().keys())
    raw = {n: reader.get(n) for n in names if n in keys and reader.kind(n) == "raw"}
    model.load_state_dict(raw, strict=False)
    if device is not None:
        model.to(device)
    if verbose:
        print(f"  loaded {len(raw)} raw tensors, replaced {replaced} Linear layers")
    return {"n_quant_replaced": replaced, "n_raw_loaded": len(raw)}
