"""GPU parity: the CUDA library against the CPU oracle and the reference goldens.

Everything here calls the library through its C ABI (directly via ctypes, or
through the drop-in optimizer classes that bind it).

Expected agreement:
  * with the oracle: bit-identical codes, scales, moments and params (both
    sides round every fp32 operation the same way, IEEE sqrt included);
  * with the reference (golden files): codes bit-identical except <= 1e-5 of
    them by one LSB, scales and params within rtol 1e-5 / atol 1e-7;
    half-precision cases within _golden.half_close (the elements torch's
    scalar tail loop rounds differently).
"""

import numpy as np
import pytest
import torch

import cases as C
from _golden import code_mismatch_fraction, golden_perms, half_close, load
from oracle import oracle
from smo_optimizer_b200 import SMO, SMO8bit, _host, _lib, ops, synthetic

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-7
CODE_FRAC = 1e-5


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    _lib.load()


TORCH_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def cuda(a, dtype="float32"):
    """Host array to the GPU; floating arrays in ``dtype`` (their values are of that dtype already)."""
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(TORCH_DTYPES[dtype]) if t.is_floating_point() else t


def host(t):
    t = t.detach()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()  # exact: every half value is an fp32 value
    return t.cpu().numpy()


# ------------------------------------------------------------------ stages

def test_synth_normal_matches_host_generator():
    for n, off in [(1, 0), (1000, 0), (12345, 77), (1 << 20, 3)]:
        ref = synthetic.synth_normal(7, 99, n, 1e-3, offset=off)
        t = torch.empty(n, dtype=torch.float32, device="cuda")
        ops.synth_normal_(t, 7, 99, 1e-3, offset=off)
        assert np.array_equal(host(t).view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("n,block", [(65536, 64), (84, 64), (100, 18), (453, 64), (7, 1), (4096, 256)])
def test_quantize_dequantize_match_oracle(n, block):
    rng = np.random.default_rng(n + block)
    x = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    x[::17] = 0.0
    q_ref, s_ref = oracle.quantize(x, block)
    q, s = ops.quantize_blockwise(cuda(x), block)
    assert np.array_equal(host(q), q_ref)
    assert np.array_equal(host(s), s_ref)
    d_ref = oracle.dequantize(q_ref, s_ref, n, block)
    d = ops.dequantize_blockwise(q, s, n, block)
    assert np.array_equal(host(d), d_ref)


@pytest.mark.parametrize("H,W,h,w,wd", [(1024, 1024, 256, 256, 0.01), (64, 64, 16, 16, 0.0), (50, 30, 12, 7, 0.01),
                                        (100, 200, 30, 60, 0.01), (33, 65, 8, 16, 0.0), (96, 96, 32, 32, 0.01)])
def test_pool_pair_matches_oracle(H, W, h, w, wd):
    g = synthetic.synth_normal(1, 1, H * W, 1e-3).reshape(H, W)
    p = synthetic.synth_normal(1, 2, H * W, 0.02).reshape(H, W)
    sc = _host.step_scalars(1e-3, (0.9, 0.999), 1e-8, wd, 1)
    ref_m, ref_2 = oracle.pool_pair(g, p, (h, w), sc)
    om, o2 = ops.pool2d_pair(cuda(g), (h, w), cuda(p), wd)
    assert np.array_equal(host(om), ref_m)
    assert np.array_equal(host(o2), ref_2)


@pytest.mark.parametrize("h,w,H,W,band", [(256, 256, 1024, 1024, 0), (16, 16, 64, 64, 0), (12, 7, 50, 30, 0),
                                          (30, 60, 100, 200, 0), (32, 64, 128, 256, 12), (202, 24, 808, 96, 3),
                                          (16, 16, 48, 48, 2), (64, 64, 64, 64, 0)])
def test_upsample_matches_oracle(h, w, H, W, band):
    src = synthetic.synth_normal(3, 5, h * w, 1.0).reshape(h, w)
    ref = oracle.upsample(src, (H, W), band)
    out = ops.upsample2d(cuda(src), (H, W), band)
    assert np.array_equal(host(out), ref)


def test_bounded_wait_times_out_and_context_survives():
    lib = _lib.load()
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    import ctypes
    st = ctypes.c_int32(-1)
    _lib.check(lib.smo_selftest_wait_timeout(ws.data_ptr(), ws.numel(), 2000, ctypes.byref(st),
                                             torch.cuda.current_stream().cuda_stream), "selftest")
    assert st.value == _lib.SMO_ERR_TIMEOUT
    # the context is still usable
    x = torch.ones(1000, device="cuda")
    assert float(x.sum().item()) == 1000.0


def test_fastmath_selftest_matches_ieee():
    """The fused step's FMA-only sqrt (every finite v >= 2^-102), reciprocal
    (every normal d in [2^-126, 2^126]) and 2^31 random in-range quotients
    equal the IEEE results bit for bit."""
    import ctypes
    lib = _lib.load()
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    counts = (ctypes.c_uint64 * 4)()
    _lib.check(lib.smo_selftest_fastmath(ws.data_ptr(), ws.numel(), 1 << 31, counts,
                                         torch.cuda.current_stream().cuda_stream), "selftest_fastmath")
    assert counts[0] == 0, f"{counts[0]} square roots differ"
    assert counts[1] == 0, f"{counts[1]} reciprocals differ"
    assert counts[2] == 0, f"{counts[2]} quotients differ"
    assert counts[3] > (1 << 31)


# ------------------------------------------------------------------ full steps

def run_gpu_case(name, steps=None, general=False):
    case = C.CASES[name]
    dt = C.case_dtype(case)
    params = [torch.nn.Parameter(cuda(a, dt)) for a in C.case_params(case)]
    groups = C.case_groups(case, params)
    cls = SMO8bit if case["opt"] == "SMO8bit" else SMO
    opt = cls(groups, **case["kwargs"])
    for p, pr in zip(params, golden_perms(name, len(params))):
        if pr is not None:  # the reference's permute_basis draws, placed before the first step
            opt.state[p]["row_perm"] = cuda(pr[0])
            opt.state[p]["col_perm"] = cuda(pr[1])
    if general:
        opt._kernel_flags = 1  # SMO_FLAG_GENERAL_PATH
    for step in range(1, (steps or case["steps"]) + 1):
        for p, g in zip(params, C.case_grads(case, step)):
            p.grad = cuda(g, dt)
        opt.step()
    torch.cuda.synchronize()
    assert opt.workspace_status() == 0, "device-side status reports a failure"
    return params, [opt.state[p] for p in params]


def run_oracle_case(name, steps=None):
    case = C.CASES[name]
    params = C.case_params(case)
    groups = C.case_groups(case, params)
    opt = oracle.OracleOptimizer(case["opt"], groups, param_dtype=C.case_dtype(case), **case["kwargs"])
    keys = [k for k, _, _ in opt.params()]
    for k, pr in zip(keys, golden_perms(name, len(keys))):
        if pr is not None:
            opt.preset_perms[k] = pr
    for step in range(1, (steps or case["steps"]) + 1):
        opt.step(C.case_grads(case, step))
    return params, [opt.state[k] for k in keys]


ALL_CASES = [n for n in C.CASES if n != "single1024"]


@pytest.mark.parametrize("name", ALL_CASES)
def test_step_bit_exact_vs_oracle(name):
    """Every case, fp32 and half precision: bit-identical to the oracle (for
    half-precision cases the fp16 eps underflow makes some parameters NaN or
    infinite, in the reference too; those match as values)."""
    gp, gs = run_gpu_case(name)
    op, os_ = run_oracle_case(name)
    dt = C.case_dtype(C.CASES[name])
    for i, (p, st, ref_p, ref_st) in enumerate(zip(gp, gs, op, os_)):
        assert p.dtype == TORCH_DTYPES[dt]
        for k in C.STATE_ARRAY_KEYS:
            if k in ref_st:
                got = host(st[k]).reshape(-1)
                ref = np.asarray(ref_st[k]).reshape(-1)
                if k in ("m_s", "v_s", "exp_avg", "exp_avg_sq"):
                    assert st[k].dtype == TORCH_DTYPES[dt], f"{name}[{i}] {k} dtype"
                assert np.array_equal(got, ref, equal_nan=got.dtype != np.int8), \
                    f"{name}[{i}] {k} differs from the oracle"
        assert np.array_equal(host(p).reshape(-1), ref_p.reshape(-1), equal_nan=True), \
            f"{name}[{i}] param differs from the oracle"


@pytest.mark.parametrize("name", ALL_CASES + ["single1024"])
def test_step_matches_reference_goldens(name):
    gp, gs = run_gpu_case(name)
    case = C.CASES[name]
    dt = C.case_dtype(case)
    gold, meta = load(name)
    stride = case.get("sample_stride")
    for i, (p, st) in enumerate(zip(gp, gs)):
        for k, v in meta["tensors"][i].items():
            got = st.get(k)
            got = list(got) if isinstance(got, tuple) else got
            assert got == v, f"{name}[{i}] state[{k!r}]"
        for k in C.STATE_ARRAY_KEYS:
            gk = f"{i}.{k}"
            assert (gk in gold) == (k in st)
            if gk not in gold:
                continue
            ref = gold[gk]
            got = host(st[k]).reshape(ref.shape)
            if dt != "float32":
                half_close(got, ref, dt, f"{name}[{i}] {k}")
            elif ref.dtype == np.int8:
                assert code_mismatch_fraction(got, ref) <= CODE_FRAC
            else:
                np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)
        flat = host(p).reshape(-1)
        if dt != "float32":
            half_close(flat[C.sample_indices(flat.size, stride)] if stride else flat,
                       gold[f"{i}.param_sample"] if stride else gold[f"{i}.param"], dt, f"{name}[{i}] param")
        elif stride:
            np.testing.assert_allclose(flat[C.sample_indices(flat.size, stride)], gold[f"{i}.param_sample"],
                                       rtol=RTOL, atol=ATOL)
        else:
            np.testing.assert_allclose(flat, gold[f"{i}.param"], rtol=RTOL, atol=ATOL)


def test_single1024_100_steps_bit_exact_vs_oracle():
    gp, gs = run_gpu_case("single1024")
    op, os_ = run_oracle_case("single1024")
    for k in ("m_q", "m_s", "v_q", "v_s"):
        assert np.array_equal(host(gs[0][k]).reshape(-1), np.asarray(os_[0][k]).reshape(-1)), k
    assert np.array_equal(host(gp[0]).reshape(-1), op[0].reshape(-1))


FUSED_CASES = ["single1024", "s8_128x256_mono", "s8_128x256_band", "s8_128x256_band_wd", "s8_multi",
               "s8_132x2048_band", "s8_256x512_k0125", "smo_96x192_k05", "smo_groups",
               "bf16_s8_mono", "bf16_s8_band_groups", "bf16_smo", "fp16_s8_groups", "fp16_s8_band", "fp16_smo"]


def bits(t):
    """A tensor's bit patterns (NaN compares equal to the same NaN)."""
    t = t.detach()
    return t.view({4: torch.int32, 2: torch.int16, 1: torch.int8}[t.element_size()])


@pytest.mark.parametrize("name", FUSED_CASES)
def test_fused_kernel_matches_general_kernels(name):
    """The fused single-pass kernel and the general two-launch kernels agree bit for bit."""
    steps = 4 if name == "single1024" else None
    fp, fs = run_gpu_case(name, steps=steps)
    gp, gs = run_gpu_case(name, steps=steps, general=True)
    for i, (a, b, sa, sb) in enumerate(zip(fp, gp, fs, gs)):
        assert torch.equal(bits(a), bits(b)), f"{name}[{i}] params differ between fused and general kernels"
        for k in C.STATE_ARRAY_KEYS:
            if k in sa:
                assert torch.equal(bits(sa[k]), bits(sb[k])), \
                    f"{name}[{i}] {k} differs between fused and general kernels"


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("H,W,k,block,band_mb,wd", [
    (4 * 33, 4 * 300, 0.25, 64, 0.0, 0.01),     # blocks straddle rows
    (4 * 40, 4 * 512, 0.25, 64, 0.25, 0.01),    # bands
    (2 * 64, 2 * 640, 0.5, 64, 0.0, 0.0),       # 2x2 windows, two cells per thread
    (8 * 24, 8 * 64, 0.125, 64, 0.0, 0.01),     # 8x8 windows (16-byte half rows)
])
def test_fused_half_precision_vs_oracle(dtype, H, W, k, block, band_mb, wd):
    """bf16 / fp16 parameters through the fused kernel (every op rounded to
    the dtype), bit-identical to the oracle over three steps."""
    kw = dict(lr=2e-3, betas=(0.9, 0.99), eps=1e-8, weight_decay=wd, k_ratio=k, block_size=block)
    if band_mb:
        kw.update(low_peak=True, band_mb=band_mb)
    std = 1e-3 if dtype == "bfloat16" else 0.05  # fp16: keep v above its underflow
    p0 = C.round_to_dtype(synthetic.synth_normal(7, H, H * W, 0.02).reshape(H, W), dtype)
    p = torch.nn.Parameter(cuda(p0, dtype))
    opt = SMO8bit([p], **kw)
    ref_p = p0.copy()
    ref = oracle.OracleOptimizer("SMO8bit", [{"params": [ref_p]}], param_dtype=dtype, **kw)
    for step in range(1, 4):
        g = C.round_to_dtype(synthetic.synth_normal(8, step * 1000 + W, H * W, std).reshape(H, W), dtype)
        p.grad = cuda(g, dtype)
        opt.step()
        ref.step([g])
    torch.cuda.synchronize()
    assert opt.workspace_status() == 0
    st, rst = opt.state[p], ref.state[(0, 0)]
    for key in ("m_q", "m_s", "v_q", "v_s"):
        got = host(st[key]).reshape(-1)
        assert np.array_equal(got, rst[key].reshape(-1), equal_nan=got.dtype != np.int8), key
    assert np.array_equal(host(p), ref_p, equal_nan=True)


@pytest.mark.parametrize("H,W,k,block,band_mb,wd", [
    (4 * 33, 4 * 300, 0.25, 64, 0.0, 0.01),     # w=300: blocks straddle rows; strips 16,16,1
    (4 * 17, 4 * 1000, 0.25, 40, 0.5, 0.0),     # w=1000 > threads: several columns per thread
    (2 * 50, 2 * 700, 0.5, 64, 0.0, 0.01),      # 2x2 windows
    (8 * 21, 8 * 40, 0.125, 20, 0.0, 0.01),     # 8x8 windows, block 20
    (32, 4 * 1024, 0.25, 64, 0.0, 0.01),        # one strip of 8 compact rows, 4 columns per thread
    (4 * 20, 4 * 1152, 0.25, 64, 0.5, 0.01),    # 384-thread CTAs, 3 columns per thread, bands
    (4 * 37, 4 * 512, 0.25, 128, 0.0, 0.0),     # 256-thread CTAs, 128-cell blocks, no weight decay
])
def test_fused_random_shapes_vs_oracle(H, W, k, block, band_mb, wd):
    kw = dict(lr=2e-3, betas=(0.8, 0.99), eps=1e-8, weight_decay=wd, k_ratio=k, block_size=block)
    if band_mb:
        kw.update(low_peak=True, band_mb=band_mb)
    p0 = synthetic.synth_normal(5, H, H * W, 0.02).reshape(H, W)
    p = torch.nn.Parameter(cuda(p0))
    opt = SMO8bit([p], **kw)
    ref_p = p0.copy()
    ref = oracle.OracleOptimizer("SMO8bit", [{"params": [ref_p]}], **kw)
    for step in range(1, 4):
        g = synthetic.synth_normal(6, step * 1000 + W, H * W, 1e-3).reshape(H, W)
        p.grad = cuda(g)
        opt.step()
        ref.step([g])
    torch.cuda.synchronize()
    assert opt.workspace_status() == 0
    st, rst = opt.state[p], ref.state[(0, 0)]
    for key in ("m_q", "m_s", "v_q", "v_s"):
        assert np.array_equal(host(st[key]).reshape(-1), rst[key].reshape(-1)), key
    assert np.array_equal(host(p), ref_p)


@pytest.mark.parametrize("eps", [1e-8, 1e-12])
def test_fused_ieee_fallback_rows_vs_oracle(eps):
    """Zero, tiny and huge gradient regions send rows of the fused kernel's
    FMA-only Adam write to its IEEE fix-up (eps < 2^-27 sends every row); the
    result stays bit-identical to the oracle."""
    H, W = 4 * 40, 4 * 384
    kw = dict(lr=1e-3, betas=(0.9, 0.999), eps=eps, weight_decay=0.01, k_ratio=0.25, block_size=64,
              low_peak=True, band_mb=0.5)
    p0 = synthetic.synth_param(8, 0, (H, W))
    p = torch.nn.Parameter(cuda(p0))
    opt = SMO8bit([p], **kw)
    ref_p = p0.copy()
    ref = oracle.OracleOptimizer("SMO8bit", [{"params": [ref_p]}], **kw)
    for step in range(1, 4):
        g = synthetic.synth_grad(8, step, 0, (H, W)).copy()
        g[8:40, :] = 0.0                      # whole zero rows: m = v = 0 there
        g[40:72, 64:512] = 0.0                # a zero patch inside rows
        g[72:104, 512:1024] *= 1e-28          # tiny: v far below 2^-100
        g[104:120, 1024:1280] *= 1e12         # huge values
        if step == 2:
            g[120:136, :256] = 0.0            # a region that turns zero later
        p.grad = cuda(g)
        opt.step()
        ref.step([g])
    torch.cuda.synchronize()
    assert opt.workspace_status() == 0
    st, rst = opt.state[p], ref.state[(0, 0)]
    for key in ("m_q", "m_s", "v_q", "v_s"):
        assert np.array_equal(host(st[key]).reshape(-1), rst[key].reshape(-1)), key
    assert np.array_equal(host(p).view(np.uint32), ref_p.view(np.uint32))


def test_fused_fp32_moments_4x4_vs_oracle():
    """SMO (fp32 pooled moments) on 4x4 windows through the fused kernel
    (384-thread CTAs, two columns per thread); bit-identical to the oracle
    over three steps."""
    H, W = 4 * 24, 4 * 768
    kw = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, k_ratio=0.25)
    p0 = synthetic.synth_param(9, 0, (H, W))
    p = torch.nn.Parameter(cuda(p0))
    opt = SMO([p], **kw)
    ref_p = p0.copy()
    ref = oracle.OracleOptimizer("SMO", [{"params": [ref_p]}], **kw)
    for step in range(1, 4):
        g = synthetic.synth_grad(9, step, 0, (H, W))
        p.grad = cuda(g)
        opt.step()
        ref.step([g])
    torch.cuda.synchronize()
    assert opt.workspace_status() == 0
    st, rst = opt.state[p], ref.state[(0, 0)]
    for key in ("exp_avg", "exp_avg_sq"):
        assert np.array_equal(host(st[key]).reshape(-1), np.asarray(rst[key]).reshape(-1)), key
    assert np.array_equal(host(p).view(np.uint32), ref_p.view(np.uint32))


def test_state_dict_round_trip_continues_bit_identically():
    """state_dict() / load_state_dict(): a run restored from a mid-run snapshot
    (into the same optimizer, and into a fresh one) continues exactly as the
    uninterrupted run, for pooled int8, dense and quant_only tensors."""
    import copy
    shapes = [(128, 512), (384, 1152), (300,), (64, 48)]
    kw = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, k_ratio=0.25, block_size=64)

    def make():
        ps = [torch.nn.Parameter(cuda(synthetic.synth_param(30, i, s))) for i, s in enumerate(shapes)]
        groups = [{"params": ps[:3]}, {"params": ps[3:], "compress": "quant_only"}]
        return ps, SMO8bit(groups, **kw)

    def run(ps, opt, steps):
        for step in steps:
            for i, (p, s) in enumerate(zip(ps, shapes)):
                p.grad = cuda(synthetic.synth_grad(30, step, i, s))
            opt.step()
        torch.cuda.synchronize()

    pa, oa = make()
    run(pa, oa, (1, 2, 3))
    snap_p = [p.detach().clone() for p in pa]
    snap_s = copy.deepcopy(oa.state_dict())
    run(pa, oa, (4, 5))
    final = [p.detach().clone() for p in pa]

    # the same optimizer, rewound
    with torch.no_grad():
        for p, s in zip(pa, snap_p):
            p.copy_(s)
    oa.load_state_dict(copy.deepcopy(snap_s))
    run(pa, oa, (4, 5))
    for i, (p, f) in enumerate(zip(pa, final)):
        assert torch.equal(p, f), f"param {i} differs after rewinding the same optimizer"

    # a fresh optimizer
    pb, ob = make()
    with torch.no_grad():
        for p, s in zip(pb, snap_p):
            p.copy_(s)
    ob.load_state_dict(copy.deepcopy(snap_s))
    run(pb, ob, (4, 5))
    for i, (p, f) in enumerate(zip(pb, final)):
        assert torch.equal(p, f), f"param {i} differs in a fresh optimizer"
    sa, sb = oa.state_dict()["state"], ob.state_dict()["state"]
    for k in sa:
        for key, v in sa[k].items():
            if torch.is_tensor(v):
                assert torch.equal(v, sb[k][key]), f"state {k}.{key} differs"
            else:
                assert v == sb[k][key], f"state {k}.{key} differs"
    assert oa.workspace_status() == 0 and ob.workspace_status() == 0


@pytest.mark.parametrize("seed", [101, 102, 103, 104])
def test_random_mixed_sets_bit_exact_vs_oracle(seed):
    """One step call over a random mix of tensor kinds and shapes: exact and
    adaptive pooled windows (fused and general kernels), row-straddling blocks,
    dense 1-D and small tensors, a quant_only group; monolithic or low_peak, or
    permute_basis; bit-identical to the oracle after three steps."""
    rng = np.random.default_rng(seed)
    shapes = []
    for _ in range(6):
        h = int(rng.integers(9, 80)) * (4 if rng.random() < 0.6 else 1) + (0 if rng.random() < 0.7 else 3)
        w = int(rng.integers(9, 180)) * (4 if rng.random() < 0.6 else 1)
        shapes.append((max(h, 33), max(w, 33)))
    shapes += [(int(rng.integers(20, 500)),), (16, 24)]
    quant_shapes = [(int(rng.integers(40, 120)), int(rng.integers(40, 120))), (int(rng.integers(50, 900)),)]
    mode = ("mono", "band", "perm", "mono")[seed % 4]
    kw = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01 if seed % 2 else 0.0, k_ratio=0.25,
              block_size=int(rng.choice([32, 64, 100])))
    if mode == "band":
        kw.update(low_peak=True, band_mb=0.05)
    if mode == "perm":
        kw.update(permute_basis=True)
    all_shapes = shapes + quant_shapes
    p0 = [synthetic.synth_param(seed, i, s) for i, s in enumerate(all_shapes)]
    ps = [torch.nn.Parameter(cuda(a)) for a in p0]
    opt = SMO8bit([{"params": ps[:len(shapes)]}, {"params": ps[len(shapes):], "compress": "quant_only"}], **kw)
    ref_p = [a.copy() for a in p0]
    ref = oracle.OracleOptimizer("SMO8bit", [{"params": ref_p[:len(shapes)]},
                                             {"params": ref_p[len(shapes):], "compress": "quant_only"}], **kw)
    keys = [k for k, _, _ in ref.params()]
    for step in range(1, 4):
        gs = [synthetic.synth_grad(seed, step, i, s) for i, s in enumerate(all_shapes)]
        for p, g in zip(ps, gs):
            p.grad = cuda(g)
        opt.step()
        if step == 1 and mode == "perm":
            # the oracle takes the permutations the library drew at its first step
            for p, k in zip(ps, keys):
                st = opt.state[p]
                if "row_perm" in st:
                    ref.preset_perms[k] = (host(st["row_perm"]), host(st["col_perm"]))
        ref.step(gs)
    torch.cuda.synchronize()
    assert opt.workspace_status() == 0
    for i, (p, k) in enumerate(zip(ps, keys)):
        st, rst = opt.state[p], ref.state[k]
        for key in C.STATE_ARRAY_KEYS:
            if key in rst:
                assert np.array_equal(host(st[key]).reshape(-1), np.asarray(rst[key]).reshape(-1)), \
                    f"tensor {i} {all_shapes[i]} state {key}"
        assert np.array_equal(host(p).view(np.uint32).reshape(-1), ref_p[i].view(np.uint32).reshape(-1)), \
            f"tensor {i} {all_shapes[i]} param"
