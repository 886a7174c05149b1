"""GPU parity: the sm_100a kernels against the oracle (itself pinned to the
reference by tests/test_oracle_golden.py) and against the reference's own
golden outputs.

Bars:
* quantize/pack: packed codes, scale/gmin, double-quant codes/meta, outlier
  indices/values, outlier tables and deltas bit-identical to the oracle;
* fused dequant-GEMM: max|y - y_ref| / max|y_ref| <= 1e-2 against the fp32
  dequant-matmul (TOL below), y_ref with exact outlier values.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import goap
from tests.conftest import golden_case_list, load_case
from tests.test_host_cpu import qt_from_case

pytestmark = pytest.mark.gpu

TOL = 1e-2  # max relative error of GEMM outputs (north star: 1e-2 vs fp32 dequant-matmul)

torch_dt = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import tensorshrink_b200._C as C
    C.load()
    yield


def dev_w(c):
    return torch.from_numpy(c["w"]).to(torch_dt[str(c["w_dtype"])]).cuda()


def dev_x(c):
    return torch.from_numpy(c["x"]).to(torch_dt[str(c["x_dtype"])]).cuda()


def mode_of(c):
    return str(c["mode"])


def quantize_case_gpu(c, **over):
    import tensorshrink_b200 as ts
    bits, gs, dq, _ = (int(v) for v in c["params"])
    mode = mode_of(c)
    kw = dict(bits=bits, group_size=gs, outlier_frac=float(c["frac"]), double_quant=bool(dq),
              companded=mode == "lloyd", nf_quant=mode == "nf")
    if mode == "lloyd":
        kw["codebook"] = torch.from_numpy(c["lloyd_cb32"])
    kw.update(over)
    return ts.quantize_device(dev_w(c), **kw)


def oracle_quantize(c, codebook=None):
    bits, gs, dq, _ = (int(v) for v in c["params"])
    mode = mode_of(c)
    cb = codebook if codebook is not None else (c["lloyd_cb32"] if mode == "lloyd" else None)
    return goap.quantize(c["w"], bits=bits, group_size=gs, outlier_frac=float(c["frac"]),
                         double_quant=bool(dq), mode=mode, codebook=cb)


def assert_device_quant_equals_oracle(d, q):
    h = lambda t: t.cpu().numpy()  # noqa: E731
    np.testing.assert_array_equal(h(d.packed), q.packed)
    np.testing.assert_array_equal(h(d.scale).view(np.uint16), q.scale.view(np.uint16))
    np.testing.assert_array_equal(h(d.gmin).view(np.uint16), q.gmin.view(np.uint16))
    if q.dq_scale_codes is not None:
        np.testing.assert_array_equal(h(d.dq_scale_codes), q.dq_scale_codes)
        np.testing.assert_array_equal(h(d.dq_gmin_codes), q.dq_gmin_codes)
        np.testing.assert_array_equal(h(d.dq_scale_meta).view(np.uint16), q.dq_scale_meta.view(np.uint16))
        np.testing.assert_array_equal(h(d.dq_gmin_meta).view(np.uint16), q.dq_gmin_meta.view(np.uint16))
    np.testing.assert_array_equal(h(d.outlier_idx), q.outlier_idx)
    np.testing.assert_array_equal(h(d.outlier_val).view(np.uint16), q.outlier_val.view(np.uint16))
    t = goap.outlier_tables(q)
    np.testing.assert_array_equal(h(d.outlier_row), t.row)
    np.testing.assert_array_equal(h(d.outlier_col), t.col)
    np.testing.assert_array_equal(h(d.outlier_delta).view(np.uint16), t.delta.view(np.uint16))
    np.testing.assert_array_equal(h(d.outlier_row_ptr), t.row_ptr)


# ---------------------------------------------------------------------------
# quantize / pack
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", golden_case_list())
def test_quantize_bit_exact(golden, name):
    c = load_case(golden, name)
    d = quantize_case_gpu(c)
    q = oracle_quantize(c)
    assert_device_quant_equals_oracle(d, q)
    # and the reference's own packed codes (tie choice cannot change codes)
    np.testing.assert_array_equal(d.packed.cpu().numpy(), c["packed"])
    if "codebook" in c:
        np.testing.assert_array_equal(d.to_quantized_tensor().codebook, c["codebook"])


@pytest.mark.parametrize("name", ["lloyd2_g64", "lloyd4_g128"])
def test_lloyd_fit_on_device(golden, name):
    """Below 300,000 values the fit uses every value, like the reference. The
    device adds each level's values in element order in float32, as the
    reference's CPU index_add_ does, so the fitted levels are the reference's
    bit for bit, and so are the codes and the stored fp16 codebook."""
    c = load_case(golden, name)
    d = quantize_case_gpu(c, codebook=None)
    cb = d.codebook_assign.cpu().numpy()
    np.testing.assert_array_equal(cb, c["lloyd_cb32"])
    assert_device_quant_equals_oracle(d, oracle_quantize(c))
    np.testing.assert_array_equal(d.packed.cpu().numpy(), c["packed"])
    np.testing.assert_array_equal(d.to_quantized_tensor().codebook, c["codebook"])


def test_lloyd_fit_standalone(golden):
    import tensorshrink_b200._C as C
    lib = C.load()
    v = torch.from_numpy(golden["lloyd/sample"]).cuda()
    for lv in (4, 16):
        out = torch.empty(lv, dtype=torch.float32, device="cuda")
        ws = torch.empty(int(lib.ts_lloyd_fit_workspace_size(v.numel(), lv)), dtype=torch.uint8, device="cuda")
        rc = lib.ts_lloyd_fit(v.data_ptr(), v.numel(), lv, 12, out.data_ptr(), ws.data_ptr(), ws.numel(),
                              torch.cuda.current_stream().cuda_stream)
        C.check(rc, "ts_lloyd_fit")
        np.testing.assert_array_equal(out.cpu().numpy(), golden[f"lloyd/cent{lv}"])


def test_lloyd_sampled_matches_oracle_fit():
    import tensorshrink_b200 as ts
    w = torch.from_numpy(goap.student_t_weights((640, 1024), seed=11)).cuda()
    g = torch.Generator(device="cuda").manual_seed(3)
    sample = torch.randperm(640 * 1024, device="cuda", generator=g)[:300_000]
    d = ts.quantize_device(w, bits=2, group_size=64, outlier_frac=0.001, companded=True, lloyd_sample=sample)
    q0 = goap.quantize(w.cpu().numpy(), bits=2, group_size=64, outlier_frac=0.001, mode="lloyd",
                       lloyd_sample=sample.cpu().numpy())
    np.testing.assert_array_equal(d.codebook_assign.cpu().numpy(), q0.assign_codebook_f32)
    assert_device_quant_equals_oracle(d, q0)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("bits,gs,mode,dq", [(4, 128, "nf", True), (2, 64, "uniform", False),
                                             (8, 128, "uniform", True), (4, 32, "uniform", False),
                                             (4, 16, "nf", False), (2, 256, "nf", True)])
def test_quantize_random_shapes(dtype, bits, gs, mode, dq):
    import tensorshrink_b200 as ts
    w = torch.from_numpy(goap.student_t_weights((137, 700), seed=bits * gs, dtype=np.float32)).to(dtype)
    d = ts.quantize_device(w.cuda(), bits=bits, group_size=gs, outlier_frac=0.002, double_quant=dq,
                           nf_quant=mode == "nf")
    wn = w.float().numpy() if dtype == torch.bfloat16 else w.numpy()
    q = goap.quantize(wn, bits=bits, group_size=gs, outlier_frac=0.002, double_quant=dq, mode=mode)
    assert_device_quant_equals_oracle(d, q)


def test_quantize_edge_cases():
    import tensorshrink_b200 as ts
    # all-equal weights: every element ties at the threshold
    w = torch.full((16, 64), 0.5, dtype=torch.float16)
    d = ts.quantize_device(w.cuda(), bits=4, group_size=64, outlier_frac=0.05)
    q = goap.quantize(w.numpy(), bits=4, group_size=64, outlier_frac=0.05)
    assert_device_quant_equals_oracle(d, q)
    assert d.outlier_idx.cpu().tolist() == list(range(51))
    # no outliers (frac 0) and k >= n
    for frac in (0.0, 1.0):
        w = torch.randn(8, 40, dtype=torch.float16)
        d = ts.quantize_device(w.cuda(), bits=2, group_size=8, outlier_frac=frac)
        q = goap.quantize(w.numpy(), bits=2, group_size=8, outlier_frac=frac)
        assert_device_quant_equals_oracle(d, q)
        assert d.outlier_idx.numel() == 0
    # single row, single group, zeros
    w = torch.zeros(1, 8, dtype=torch.float16)
    d = ts.quantize_device(w.cuda(), bits=8, group_size=8, outlier_frac=0.2)
    q = goap.quantize(w.numpy(), bits=8, group_size=8, outlier_frac=0.2)
    assert_device_quant_equals_oracle(d, q)


# ---------------------------------------------------------------------------
# fused dequant-GEMM
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", golden_case_list())
def test_qlinear_matches_reference_outputs(golden, name):
    import tensorshrink_b200 as ts
    c = load_case(golden, name)
    bias = torch.from_numpy(c["bias"]).to(torch_dt[str(c["x_dtype"])]) if "bias" in c else None
    ql = ts.QuantLinear(qt_from_case(c), bias).cuda()
    y = ql(dev_x(c))
    assert y.dtype == torch_dt[str(c["x_dtype"])]
    err = goap.max_rel_error(y.float().cpu().numpy(), c["y_ref"])
    assert err <= TOL, err


def _random_layer(rows, cols, bits, gs, mode, dq, seed, frac=0.002):
    import tensorshrink_b200 as ts
    w = torch.from_numpy(goap.student_t_weights((rows, cols), seed=seed)).cuda()
    d = ts.quantize_device(w, bits=bits, group_size=gs, outlier_frac=frac, double_quant=dq,
                           nf_quant=mode == "nf")
    return d


@pytest.mark.parametrize("bits,gs,mode,dq", [(4, 128, "nf", True), (4, 128, "uniform", False),
                                             (4, 64, "nf", False), (2, 64, "uniform", False),
                                             (2, 128, "nf", True), (8, 128, "uniform", True),
                                             (8, 64, "nf", False), (4, 32, "uniform", True),
                                             (4, 16, "uniform", False)])
@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16])
def test_qlinear_random_shapes(bits, gs, mode, dq, xdt):
    import tensorshrink_b200 as ts
    rows, cols = 301, 1000
    d = _random_layer(rows, cols, bits, gs, mode, dq, seed=bits * 1000 + gs)
    bias = (torch.randn(rows) * 0.1).to(xdt).cuda()
    ql = ts.QuantLinear.from_device_quant(d, bias)
    q = d.to_quantized_tensor()
    W = goap.dequantize(q)
    g = torch.Generator().manual_seed(5)
    for M in (1, 2, 3, 4, 5, 8, 9, 16, 33, 64, 100):
        x = torch.randn((M, cols), generator=g).to(xdt)
        y = ql(x.cuda()).float().cpu().numpy()
        ref = x.float().numpy() @ W.T + bias.float().cpu().numpy()
        err = goap.max_rel_error(y, ref)
        assert err <= TOL, (M, err)


def test_qlinear_config1_full_size():
    """Config 1: 4096x4096, 4-bit g128, double-quant, NF4, outlier_frac 1e-3."""
    import tensorshrink_b200 as ts
    w = torch.from_numpy(goap.student_t_weights((4096, 4096), seed=1)).cuda()
    d = ts.quantize_device(w, bits=4, group_size=128, outlier_frac=0.001, double_quant=True, nf_quant=True)
    q = goap.quantize(w.cpu().numpy(), bits=4, group_size=128, outlier_frac=0.001, double_quant=True, mode="nf")
    assert_device_quant_equals_oracle(d, q)
    assert d.outlier_idx.numel() == 16777
    ql = ts.QuantLinear.from_device_quant(d)
    W = goap.dequantize(q)
    for M in (1, 16):
        x = torch.randn(M, 4096, dtype=torch.float16)
        y = ql(x.cuda()).float().cpu().numpy()
        err = goap.max_rel_error(y, x.float().numpy() @ W.T)
        assert err <= TOL, (M, err)


@pytest.mark.parametrize("shape", [(14336, 4096), (4096, 14336)])
def test_qlinear_mlp_shapes(shape):
    """Config 2 matrices: 4-bit g128 uniform + outliers, bf16 activations."""
    import tensorshrink_b200 as ts
    d = _random_layer(*shape, bits=4, gs=128, mode="uniform", dq=False, seed=shape[0], frac=0.001)
    ql = ts.QuantLinear.from_device_quant(d)
    W = goap.dequantize(d.to_quantized_tensor())
    for M in (1, 8, 32, 64):
        x = torch.randn(M, shape[1]).to(torch.bfloat16)
        y = ql(x.cuda()).float().cpu().numpy()
        err = goap.max_rel_error(y, x.float().numpy() @ W.T)
        assert err <= TOL, (M, err)


@pytest.mark.parametrize("rows,cols,bits,mode", [(256, 16384, 4, "uniform"), (256, 16384, 4, "nf"),
                                                 (200, 32768, 2, "uniform")])
def test_qlinear_split_row_blocks(rows, cols, bits, mode):
    """Few row blocks of four tiles each: the decode kernel splits row blocks
    between CTAs and finishes them through the workspace partial sums."""
    import tensorshrink_b200 as ts
    d = _random_layer(rows, cols, bits=bits, gs=128, mode=mode, dq=False, seed=rows + bits, frac=0.001)
    ql = ts.QuantLinear.from_device_quant(d)
    W = goap.dequantize(d.to_quantized_tensor())
    for M in (1, 5, 8):
        x = torch.randn(M, cols).to(torch.bfloat16)
        y = ql(x.cuda()).float().cpu().numpy()
        err = goap.max_rel_error(y, x.float().numpy() @ W.T)
        assert err <= TOL, (M, err)


@pytest.mark.parametrize("mode", ["uniform", "nf"])
def test_qlinear_many_outliers(mode):
    """2% outliers: a CTA's outlier slice exceeds the preloaded part, the rest
    is read in place."""
    import tensorshrink_b200 as ts
    d = _random_layer(2048, 4096, bits=4, gs=128, mode=mode, dq=False, seed=77, frac=0.02)
    ql = ts.QuantLinear.from_device_quant(d)
    W = goap.dequantize(d.to_quantized_tensor())
    for M in (1, 3, 8):
        x = torch.randn(M, 4096).to(torch.bfloat16)
        y = ql(x.cuda()).float().cpu().numpy()
        err = goap.max_rel_error(y, x.float().numpy() @ W.T)
        assert err <= TOL, (M, err)


def test_functional_api_unsorted_outliers_and_fp32():
    import tensorshrink_b200 as ts
    from tensorshrink_b200.kernels import fused_quantized_linear
    d = _random_layer(257, 512, 4, 128, "nf", True, seed=9)
    q = d.to_quantized_tensor()
    W = goap.dequantize(q)
    x = torch.randn(3, 512, dtype=torch.float16)
    perm = torch.randperm(d.outlier_row.numel(), device="cuda")
    common = dict(x=x.cuda(), packed=d.packed, scale=None, gmin=None, bias=None, bits=4, group_size=128,
                  cols=512, out_features=257, compute_dtype=torch.float16,
                  codebook=d.codebook_store.float(), dq_scale_codes=d.dq_scale_codes,
                  dq_scale_meta=d.dq_scale_meta, dq_gmin_codes=d.dq_gmin_codes,
                  dq_gmin_meta=d.dq_gmin_meta, dq_group_size=256, n_groups=4)
    y1 = fused_quantized_linear(**common, outlier_row=d.outlier_row[perm], outlier_col=d.outlier_col[perm],
                                outlier_delta=d.outlier_delta[perm], outliers_sorted=False, return_fp32=True)
    y2 = fused_quantized_linear(**common, outlier_row=d.outlier_row, outlier_col=d.outlier_col,
                                outlier_delta=d.outlier_delta)
    assert y1.dtype == torch.float32 and y2.dtype == torch.float16
    ref = x.float().numpy() @ W.T
    assert goap.max_rel_error(y1.cpu().numpy(), ref) <= TOL
    assert goap.max_rel_error(y2.float().cpu().numpy(), ref) <= TOL


def test_dequantize_weight_and_outlier_pass():
    import tensorshrink_b200 as ts
    from tensorshrink_b200.kernels import apply_outlier_correction
    d = _random_layer(130, 384, 2, 64, "uniform", True, seed=4)
    ql = ts.QuantLinear.from_device_quant(d)
    Wd = ql.dequantize(torch.float32).cpu().numpy()
    q = d.to_quantized_tensor()
    Wo = goap.dequantize(q)
    # outlier positions hold base + fp16(delta): within fp16 rounding of the exact value
    np.testing.assert_allclose(Wd, Wo, rtol=2e-3, atol=2e-6)
    Wbase = goap.dequantize(q, exact_outliers=False)
    mask = np.ones_like(Wbase, dtype=bool)
    mask.reshape(-1)[q.outlier_idx] = False
    np.testing.assert_array_equal(Wd[mask], Wbase[mask])
    # standalone atomic correction adds x[:,col]*delta
    x = torch.randn(4, 384, dtype=torch.float16).cuda()
    out = torch.zeros(4, 130, dtype=torch.float32, device="cuda")
    apply_outlier_correction(out, x, d.outlier_row, d.outlier_col, d.outlier_delta)
    ref = np.zeros((4, 130), np.float32)
    xr = x.float().cpu().numpy()
    for r, cidx, dl in zip(d.outlier_row.cpu().numpy(), d.outlier_col.cpu().numpy(),
                           d.outlier_delta.float().cpu().numpy()):
        ref[:, r] += xr[:, cidx] * dl
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-6)


def test_dequantize_tensor_matches_oracle(golden):
    import tensorshrink_b200 as ts
    for name in ("nf4_dq_g128", "lloyd2_g64", "u8_dq_g128"):
        c = load_case(golden, name)
        qt = qt_from_case(c)
        W = ts.dequantize_tensor(qt, dtype=torch.float32).numpy()
        np.testing.assert_array_equal(W, goap.dequantize(qt))


def test_qlinear_deterministic_and_graph_capturable():
    import tensorshrink_b200 as ts
    d = _random_layer(4096, 4096, 4, 128, "nf", True, seed=2)
    ql = ts.QuantLinear.from_device_quant(d)
    x = torch.randn(1, 4096, dtype=torch.float16, device="cuda")
    y0 = ql(x)
    for _ in range(3):
        assert torch.equal(ql(x), y0)
    static_x = x.clone()
    ql(static_x)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        static_y = ql(static_x)
    x2 = torch.randn(1, 4096, dtype=torch.float16, device="cuda")
    static_x.copy_(x2)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(static_y, ql(x2))


def test_quantize_module_end_to_end():
    """quantize_module swaps the Linears; the quantized model's output matches
    the same model run with the layers' dequantized fp32 weights."""
    import tensorshrink_b200 as ts
    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(512, 1024), torch.nn.SiLU(), torch.nn.Linear(1024, 512)).cuda().half()
    x = torch.randn(4, 512, dtype=torch.float16, device="cuda")
    stats = ts.quantize_module(m, bits=8, verbose=False)
    assert stats["n_replaced"] == 2 and isinstance(m[0], ts.QuantLinear) and isinstance(m[2], ts.QuantLinear)
    assert all(layer["rel_error"] < 0.05 for layer in stats["layers"])
    with torch.no_grad():
        y = m(x).float()
        h = torch.nn.functional.silu(x.float() @ m[0].dequantize().T + m[0].bias.float())
        ref = h.half().float() @ m[2].dequantize().T + m[2].bias.float()
    assert goap.max_rel_error(y.cpu().numpy(), ref.cpu().numpy()) <= TOL


def test_errors_are_loud():
    import tensorshrink_b200 as ts
    d = _random_layer(64, 256, 4, 128, "uniform", False, seed=1)
    ql = ts.QuantLinear.from_device_quant(d)
    with pytest.raises(RuntimeError):
        ql(torch.randn(1, 256, dtype=torch.float16))          # CPU input
    from tensorshrink_b200.kernels import fused_quantized_linear
    with pytest.raises(NotImplementedError):
        fused_quantized_linear(torch.randn(1, 256, device="cuda"), d.packed, d.scale, d.gmin, None, 6, 128,
                               256, 64, torch.float16)
    with pytest.raises(NotImplementedError):
        ts.quantize_device(torch.randn(8, 64, device="cuda"), bits=4, group_size=48)


def test_workspace_shared_across_shapes():
    """One cached workspace serves weights of different row counts in any
    order (the layout does not depend on the weight's shape)."""
    import tensorshrink_b200 as ts
    layers = [_random_layer(r, c, 4, 128, "uniform", False, seed=r + c) for r, c in
              ((512, 4096), (14336, 4096), (4096, 14336), (1000, 2048))]
    qls = [ts.QuantLinear.from_device_quant(d) for d in layers]
    Ws = [torch.from_numpy(goap.dequantize(d.to_quantized_tensor())).cuda() for d in layers]
    g = torch.Generator(device="cuda").manual_seed(3)
    for rnd in range(3):
        for i in ((0, 1, 2, 3), (3, 2, 1, 0), (1, 0, 2, 0))[rnd]:
            M = (1, 8, 3)[rnd]
            x = torch.randn(M, qls[i].in_features, device="cuda", generator=g).to(torch.bfloat16)
            y = qls[i](x).float()
            ref = x.float() @ Ws[i].T
            err = ((y - ref).abs().max() / ref.abs().max()).item()
            assert err <= TOL, (rnd, i, err)
