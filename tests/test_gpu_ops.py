"""GPU parity of the op-level C ABI against the CPU oracle.

Tolerances: f32-accumulate results within 1e-3 max
relative error (max|gpu - ref| / max|ref|); integer work bit-exact.  The int8
GEMV is additionally held to 2e-5, its measured accuracy, so that a
regression in the fixed-point path shows up long before the contract bound.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from esolearn_b200 import QuantLinear, QWeight, matmul_i8_f32
from esolearn_b200 import _native as N
from tests.gpu_util import rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL_F32 = 1e-3
TOL_GEMV = 2e-5


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def vp(t):
    return C.c_void_p(t.data_ptr())


@pytest.fixture(scope="module", autouse=True)
def _init():
    N.check(N.lib().sb_init(0))


@pytest.mark.parametrize("M", [1, 2, 3, 4, 7])
@pytest.mark.parametrize("K,N_", [(512, 1536), (4096, 4096), (1376, 512), (100, 45), (16, 16), (4096, 32000)])
def test_matmul_i8_f32_per_tensor(M, K, N_):
    rng = np.random.default_rng(M * 1000 + K + N_)
    w = (rng.standard_normal((K, N_)) * 0.02).astype(np.float32)
    q, s = O.quantize_symmetric(w)
    q = q.reshape(K, N_)
    a = rng.standard_normal((M, K)).astype(np.float32)
    ref = O.matmul_i8_f32(a, q, s, M, K, N_)
    qw = QWeight(q, [s])
    out = matmul_i8_f32(dev(a), qw).cpu().numpy()
    torch.cuda.synchronize()
    e = rel_err(out, ref)
    assert e < TOL_F32 and e < TOL_GEMV, e


@pytest.mark.parametrize("M", [5, 8, 17, 32])
@pytest.mark.parametrize("K,N_", [(4096, 4096), (11008, 4096), (4096, 11008), (512, 1536), (96, 384), (100, 45)])
@pytest.mark.parametrize("bf16", [False, True])
def test_batched_tensor_core_matmul_equals_rowwise_gemv(M, K, N_, bf16):
    # 5-32 rows of a 128-column-tile weight run on the tcgen05 tensor cores
    # with the GEMV's fixed-point arithmetic: every row must equal the GEMV of
    # that row alone bit for bit, and the reference within the f32 bar.
    # (K=100 is not a multiple of 32: that case runs the GEMV 4 rows at a time.)
    rng = np.random.default_rng(M * 7919 + K + N_ + bf16)
    w = (rng.standard_normal((K, N_)) * 0.02).astype(np.float32)
    q, s = O.quantize_symmetric(w)
    q = q.reshape(K, N_)
    a = rng.standard_normal((M, K)).astype(np.float32)
    qw = QWeight(q, [s], tile_n=128)
    at = torch.from_numpy(a).cuda()
    if bf16:
        at = at.to(torch.bfloat16)
        a = at.float().cpu().numpy()
    out = matmul_i8_f32(at, qw).cpu().numpy()
    rows = np.vstack([matmul_i8_f32(at[i:i + 1].contiguous(), qw).cpu().numpy() for i in range(M)])
    torch.cuda.synchronize()
    assert np.array_equal(out, rows)
    ref = O.matmul_i8_f32(a, q, s, M, K, N_)
    assert rel_err(out, ref) < TOL_F32


@pytest.mark.parametrize("M", [33, 48, 64])
@pytest.mark.parametrize("K,N_", [(4096, 4096), (512, 1536), (20480, 256), (96, 384)])
def test_batched_tensor_core_matmul_33_to_64_rows(M, K, N_):
    # 33-64 rows: the MMA's B operand grows to 3M+1 plane rows (up to 208),
    # stages hold one unit and TMEM is drained in two passes; K beyond 16384
    # keeps the int32 accumulators exact.  Bit-equal to row-wise GEMVs.
    rng = np.random.default_rng(M * 131 + K + N_)
    w = (rng.standard_normal((K, N_)) * 0.02).astype(np.float32)
    q, s = O.quantize_symmetric(w)
    q = q.reshape(K, N_)
    a = rng.standard_normal((M, K)).astype(np.float32)
    qw = QWeight(q, [s], tile_n=128)
    at = torch.from_numpy(a).cuda()
    out = matmul_i8_f32(at, qw).cpu().numpy()
    rows = np.vstack([matmul_i8_f32(at[i:i + 1].contiguous(), qw).cpu().numpy() for i in range(M)])
    torch.cuda.synchronize()
    assert np.array_equal(out, rows)
    ref = O.matmul_i8_f32(a, q, s, M, K, N_)
    assert rel_err(out, ref) < TOL_F32


@pytest.mark.parametrize("M", [65, 128, 200])
@pytest.mark.parametrize("K,N_", [(4096, 4096), (4096, 11008), (512, 1536)])
@pytest.mark.parametrize("bf16", [False, True])
def test_matmul_beyond_64_rows_runs_in_tensor_core_chunks(M, K, N_, bf16):
    # More than 64 rows: balanced chunks of 33-64 rows, one tensor-core GEMM
    # each, sharing one workspace in stream order.  Bit-equal to row-wise
    # GEMVs (rows are independent), within the f32 bar of the oracle.
    rng = np.random.default_rng(M * 7 + K + N_ + bf16)
    w = (rng.standard_normal((K, N_)) * 0.02).astype(np.float32)
    q, s = O.quantize_symmetric(w)
    q = q.reshape(K, N_)
    at = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32))
    if bf16:
        at = at.to(torch.bfloat16)
    a = at.float().numpy()
    at = at.cuda()
    qw = QWeight(q, [s], tile_n=128)
    out = matmul_i8_f32(at, qw).cpu().numpy()
    rows = np.vstack([matmul_i8_f32(at[i:i + 1].contiguous(), qw).cpu().numpy() for i in range(M)])
    torch.cuda.synchronize()
    assert np.array_equal(out, rows)
    assert rel_err(out, O.matmul_i8_f32(a, q, s, M, K, N_)) < TOL_F32


@pytest.mark.parametrize("M", [1, 2, 3, 4])
@pytest.mark.parametrize("K,N_,bf16,bias", [(4096, 4096, True, False), (11008, 4096, True, False),
                                             (4096, 11008, False, True), (1000, 640, False, False),
                                             (4096, 32000, True, True)])
def test_split_k_gemv_equals_one_cta_per_tile_gemv(M, K, N_, bf16, bias):
    # 1-4 rows of a 128-column-tile weight with fewer tiles than SMs take the
    # split-K GEMV (CTA per (tile, k range), int64 sums, the tile's last split
    # applies the epilogue); its output must equal bit for bit the one-CTA-per-
    # tile GEMV on the same int8 values (a narrower tiling, below), and the
    # oracle within the GEMV bar.  4096 x 32000 (250 tiles) stays on the plain
    # GEMV.  K = 1000 ends in a partial k-step.
    rng = np.random.default_rng(M + K + N_)
    q = rng.integers(-127, 128, (K, N_), dtype=np.int8)
    s = np.float32(1.3e-4)
    x = rng.standard_normal((M, K)).astype(np.float32)
    if bf16:
        xt = torch.from_numpy(x).to(torch.bfloat16)
        x = xt.float().numpy()
        xd = xt.cuda()
    else:
        xd = dev(x)
    b = rng.standard_normal(N_).astype(np.float32) if bias else None
    ref = O.matmul_i8_f32(x, q, s, M, K, N_) + (b[None, :] if bias else 0)
    wide = QWeight(q, s, tile_n=128)
    narrow = QWeight(q, s, tile_n=16)
    kw = {"bias": dev(b)} if bias else {}
    out = matmul_i8_f32(xd, wide, **kw).cpu().numpy()
    assert np.array_equal(out, matmul_i8_f32(xd, narrow, **kw).cpu().numpy())
    assert np.array_equal(out, matmul_i8_f32(xd, wide, **kw).cpu().numpy())  # the workspace was left clean
    assert rel_err(out, ref) < TOL_GEMV


@pytest.mark.parametrize("group", [32, 64])
@pytest.mark.parametrize("M", [1, 4, 8, 32, 128])
@pytest.mark.parametrize("K,N_", [(4096, 4096), (11008, 4096), (4096, 11008), (4096, 32000)])
def test_matmul_grouped_bf16_sweep_shapes(group, M, K, N_):
    # Quantized-linear sweep inputs: int8 uniform in [-127,127], f32 group
    # scales = absmax/127 of N(0,0.02) groups, bf16 activations ~ N(0,1).
    rng = np.random.default_rng(K + N_ + group + M)
    q = rng.integers(-127, 128, (K, N_), dtype=np.int8)
    src = (rng.standard_normal((K // group, group, N_)) * 0.02).astype(np.float32)
    scales = (np.abs(src).max(axis=1) / np.float32(127.0)).astype(np.float32)
    a16 = torch.randn(M, K, generator=torch.Generator().manual_seed(M + K)).to(torch.bfloat16)
    a32 = a16.float().numpy()
    ref = O.matmul_i8_f32_grouped(a32, q, scales, group, M, K, N_)
    qw = QWeight(q, scales, group=group)
    out = matmul_i8_f32(a16.cuda(), qw).cpu().numpy()
    assert rel_err(out, ref) < TOL_GEMV
    # 128-column tiles: 5+ rows take the tensor-core path (one accumulator per
    # group, chunks of at most 32 rows), 1-4 rows the GEMV
    qt = QWeight(q, scales, group=group, tile_n=128)
    out_t = matmul_i8_f32(a16.cuda(), qt).cpu().numpy()
    assert rel_err(out_t, ref) < TOL_GEMV
    again = matmul_i8_f32(a16.cuda(), qt).cpu().numpy()
    assert np.array_equal(again, out_t)  # deterministic: pieces are added in a fixed order


@pytest.mark.parametrize("M", [5, 17, 32, 33, 77])
@pytest.mark.parametrize("group", [32, 64])
def test_grouped_tensor_core_rows_and_bias(M, group):
    # Row counts around the 32-row chunking, with the bias epilogue (QuantLinear
    # with group scales), against the derived grouped oracle.
    rng = np.random.default_rng(M * 3 + group)
    K, N_ = 1024, 640
    q = rng.integers(-127, 128, (K, N_), dtype=np.int8)
    scales = (rng.random((K // group, N_)) * 1e-3 + 1e-4).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = rng.standard_normal(N_).astype(np.float32)
    ref = O.matmul_i8_f32_grouped(x, q, scales, group, M, K, N_) + bias[None, :]
    qt = QWeight(q, scales, group=group, tile_n=128)
    out = matmul_i8_f32(dev(x), qt, bias=dev(bias)).cpu().numpy()
    assert rel_err(out, ref) < TOL_GEMV


@pytest.mark.parametrize("seq", [1, 3, 77, 200])
@pytest.mark.parametrize("fin,fout", [(768, 2304), (768, 3072), (3072, 768), (512, 2048), (2048, 512)])
def test_quant_linear_forward_matches_reference_linear(seq, fin, fout):
    # nn::linear::Linear after quantize_weights() (linear.rs:56-95), the layer
    # of the other quantize consumers: GPT-2 (768 -> 2304 / 3072, 3072 -> 768)
    # and Whisper-base MLP (512 <-> 2048) shapes; 1-3 rows on the GEMV, 77 and
    # 200 on the tensor cores (200 in four chunks), all with the bias epilogue.
    rng = np.random.default_rng(seq + fin + fout)
    w = (rng.standard_normal((fin, fout)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(fout) * 0.1).astype(np.float32)
    lin = QuantLinear(w, b)
    q, s = O.quantize_symmetric(w)
    assert lin.scale == s and np.array_equal(lin.weight_q.ravel(), q)
    x = rng.standard_normal((seq, fin)).astype(np.float32)
    out = lin(dev(x)).cpu().numpy()
    ref = O.matmul_i8_f32(x, q.reshape(fin, fout), s, seq, fin, fout) + b  # cpu.rs:554-570
    assert rel_err(out, ref) < TOL_F32


def test_matmul_bias_and_zero_weights():
    rng = np.random.default_rng(7)
    K, N_, M = 256, 96, 3
    a = rng.standard_normal((M, K)).astype(np.float32)
    bias = rng.standard_normal(N_).astype(np.float32)
    q = np.zeros((K, N_), np.int8)
    qw = QWeight(q, [0.0])
    out = matmul_i8_f32(dev(a), qw, bias=dev(bias)).cpu().numpy()
    assert np.array_equal(out, np.broadcast_to(bias, (M, N_)))
    w = (rng.standard_normal((K, N_)) * 0.02).astype(np.float32)
    q, s = O.quantize_symmetric(w)
    q = q.reshape(K, N_)
    qw = QWeight(q, [s])
    ref = O.matmul_i8_f32(a, q, s, M, K, N_) + bias  # cpu.rs:554-570
    out = matmul_i8_f32(dev(a), qw, bias=dev(bias)).cpu().numpy()
    assert rel_err(out, ref) < TOL_GEMV


def test_matmul_zero_and_tiny_activations():
    rng = np.random.default_rng(8)
    K, N_ = 512, 64
    q = rng.integers(-127, 128, (K, N_), dtype=np.int8)
    qw = QWeight(q, [0.01])
    a = np.zeros((2, K), np.float32)
    a[1, 3] = 1e-30  # a single denormal-range value must not break the exponent choice
    out = matmul_i8_f32(dev(a), qw).cpu().numpy()
    ref = O.matmul_i8_f32(a, q, 0.01, 2, K, N_)
    assert np.array_equal(out[0], np.zeros(N_, np.float32))
    assert rel_err(out[1], ref[1]) < TOL_GEMV


def test_rmsnorm_matches_reference():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 4096)).astype(np.float32)
    w = rng.standard_normal(4096).astype(np.float32)
    ref = O.rmsnorm(x, w, 1e-5)
    xd, wd = dev(x), dev(w)
    out = torch.empty_like(xd)
    N.check(N.lib().sb_rmsnorm(vp(xd), vp(wd), 5, 4096, 1e-5, vp(out), None))
    torch.cuda.synchronize()
    d = np.abs(out.cpu().numpy().view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    assert d.max() <= 1  # f64 row sum in a different order: at most 1 ulp in f32


@pytest.mark.parametrize("scale", [1.0, 0.125])
def test_rope_matches_reference(scale):
    rng = np.random.default_rng(4)
    seq, heads, hd, start = 3, 8, 64, 37
    x = rng.standard_normal(seq * heads * hd).astype(np.float32)
    fr = O.compute_rope_freqs(hd, 10000.0).astype(np.float32)
    ref = O.scale(O.rope(x, seq, heads, hd, start, fr), scale)
    xd, fd = dev(x), dev(fr)
    out = torch.empty_like(xd)
    N.check(N.lib().sb_rope_with_freqs(vp(xd), seq, heads, hd, start, vp(fd), scale, vp(out), None))
    torch.cuda.synchronize()
    d = np.abs(out.cpu().numpy().view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    assert d.max() <= 1


def test_swiglu_matches_reference():
    rng = np.random.default_rng(5)
    g = rng.standard_normal(11008).astype(np.float32) * 3
    u = rng.standard_normal(11008).astype(np.float32)
    ref = O.swiglu(g, u)
    gd, ud = dev(g), dev(u)
    out = torch.empty_like(gd)
    N.check(N.lib().sb_swiglu(vp(gd), vp(ud), g.size, vp(out), None))
    torch.cuda.synchronize()
    d = np.abs(out.cpu().numpy().view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    assert d.max() <= 1


def test_argmax_rows_ties_to_last():
    x = np.zeros((3, 32000), np.float32)
    x[0, [5, 77, 31999]] = 2.0
    x[1, 0] = 1.0
    x[2, [100, 200]] = -1.0
    x[2] -= 5.0
    xd = dev(x)
    out = torch.empty(3, dtype=torch.int32, device="cuda")
    N.check(N.lib().sb_argmax_rows(vp(xd), 3, 32000, vp(out), None))
    got = out.cpu().numpy().tolist()
    assert got == [O.argmax(x[i]) for i in range(3)] == [31999, 0, 31999]


def test_device_quantizer_bit_exact():
    rng = np.random.default_rng(6)
    w = (rng.standard_normal(1 << 20) * 0.02).astype(np.float32)
    w[1234] = 0.5  # exact .5 products exercise round-half-away-from-zero
    qo, so = O.quantize_symmetric(w)
    wd = dev(w)
    q = torch.empty(w.size, dtype=torch.int8, device="cuda")
    s = torch.empty(1, dtype=torch.float32, device="cuda")
    N.check(N.lib().sb_quantize_symmetric(vp(wd), w.size, vp(q), vp(s), None))
    torch.cuda.synchronize()
    assert s.item() == so
    assert np.array_equal(q.cpu().numpy(), qo)


@pytest.mark.parametrize("vals,q,scale", [
    ([float("nan"), 1.0, -3.0], [0, 42, -127], np.float32(3.0) / np.float32(127.0)),
    ([float("inf"), 1.0, -2.0], [0, 0, 0], np.float32("inf")),
    ([float("nan"), float("nan")], [0, 0], np.float32(0.0)),
    ([1e-45, -1e-45], [127, -127], np.float32(0.0)),
])
def test_device_quantizer_special_values(vals, q, scale):
    # Rust's float rules where quantize.rs meets non-finite weights: the
    # absmax fold skips NaN, f32::clamp keeps NaN and `as i8` makes it 0.
    w = np.array(vals, np.float32)
    qo, so = O.quantize_symmetric(w)
    assert np.ravel(qo).tolist() == q
    wd = dev(w)
    qd = torch.empty(w.size, dtype=torch.int8, device="cuda")
    sd = torch.empty(1, dtype=torch.float32, device="cuda")
    N.check(N.lib().sb_quantize_symmetric(vp(wd), w.size, vp(qd), vp(sd), None))
    torch.cuda.synchronize()
    assert qd.cpu().numpy().tolist() == q
    assert sd.cpu().numpy().tobytes() == np.array([scale], np.float32).tobytes()


def _paged(cache_rows, page_size, n_kv, hd, perm, total_pages):
    """Scatter contiguous [S, n_kv*hd] rows into pages [P][n_kv][page][hd] via a page table."""
    S = cache_rows.shape[0]
    npages = (S + page_size - 1) // page_size
    pages = np.zeros((total_pages, n_kv, page_size, hd), np.float32)
    table = np.zeros(npages, np.int32)
    for i in range(npages):
        table[i] = perm[i]
        rows = cache_rows[i * page_size:(i + 1) * page_size].reshape(-1, n_kv, hd)
        pages[perm[i], :, :rows.shape[0], :] = rows.transpose(1, 0, 2)
    return pages, table


@pytest.mark.parametrize("kv_dtype", ["f32", "bf16"])
@pytest.mark.parametrize("n_q,n_kv,hd", [(8, 8, 64), (32, 8, 128), (64, 8, 128), (4, 2, 64), (32, 32, 128)])
def test_paged_gqa_decode_attention(kv_dtype, n_q, n_kv, hd):
    rng = np.random.default_rng(n_q * 7 + hd)
    B, page = 3, 16
    lens = [1, 37, 300]  # ragged contexts, including a single position and partial pages
    max_pages = (max(lens) + page - 1) // page
    q = (rng.standard_normal((B, n_q * hd)) / np.sqrt(hd)).astype(np.float32)
    all_pages, tables, refs = [], [], []
    perm = rng.permutation(B * max_pages)
    kps, vps = np.zeros((B * max_pages, n_kv, page, hd), np.float32), np.zeros((B * max_pages, n_kv, page, hd), np.float32)
    for b, S in enumerate(lens):
        k = rng.standard_normal((S, n_kv * hd)).astype(np.float32)
        v = rng.standard_normal((S, n_kv * hd)).astype(np.float32)
        if kv_dtype == "bf16":
            k, v = O.round_bf16(k), O.round_bf16(v)
        myperm = perm[b * max_pages:(b + 1) * max_pages]
        kp, tab = _paged(k, page, n_kv, hd, myperm, B * max_pages)
        vp_, _ = _paged(v, page, n_kv, hd, myperm, B * max_pages)
        kps += kp
        vps += vp_
        t = np.zeros(max_pages, np.int32)
        t[:len(tab)] = tab
        tables.append(t)
        refs.append(O.attention_decode(q[b], k, v, n_q, n_kv, hd))
    if kv_dtype == "bf16":
        kd, vd = dev(kps).to(torch.bfloat16), dev(vps).to(torch.bfloat16)
        kvt = N.SB_KV_BF16
    else:
        kd, vd = dev(kps), dev(vps)
        kvt = N.SB_KV_F32
    qd = dev(q)
    td = dev(np.stack(tables))
    ld = dev(np.array(lens, np.int32))
    out = torch.empty_like(qd)
    N.check(N.lib().sb_attn_decode_paged(vp(qd), vp(kd), vp(vd), kvt, vp(td), max_pages, vp(ld), B, n_q, n_kv, hd,
                                         page, max_pages * page, vp(out), None))
    got = out.cpu().numpy()
    for b in range(B):
        assert rel_err(got[b], refs[b]) < 1e-5, b


@pytest.mark.parametrize("m", [1, 3, 8, 64, 100])
def test_i8_storage_matmul_as_the_reference_trait_calls_it(m):
    # MathBackend::matmul_i8_f32(a, b_q, scale, m, k, n) (backend/mod.rs:521-533)
    # with b_q from i8_from_vec(Vec<i8>) -- no shape until the call -- and the
    # scale passed per call; the _bias form adds bias[n] (mod.rs:537-557).
    from esolearn_b200 import B200Backend

    rng = np.random.default_rng(m)
    k, n = 512, 384
    q = rng.integers(-127, 128, (k, n), dtype=np.int8)
    b_q = B200Backend.i8_from_vec(q.ravel())
    assert np.array_equal(B200Backend.i8_to_vec(b_q), q.ravel())
    a = rng.standard_normal((m, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    for scale in (np.float32(0.0123), np.float32(0.5)):
        got = B200Backend.matmul_i8_f32(dev(a), b_q, scale, m, k, n).cpu().numpy()
        assert rel_err(got, O.matmul_i8_f32(a, q, scale, m, k, n)) < 2e-5
        gb = B200Backend.matmul_i8_f32_bias(dev(a), b_q, scale, dev(bias), m, k, n).cpu().numpy()
        assert rel_err(gb, O.matmul_i8_f32(a, q, scale, m, k, n) + bias[None, :]) < 2e-5
    # another view of the same bytes (the storage has no shape of its own)
    q2 = q.ravel()[: 256 * 768].reshape(256, 768)
    got2 = B200Backend.matmul_i8_f32(dev(np.ascontiguousarray(a[:, :256])), b_q, np.float32(0.02), m, 256, 768)
    assert rel_err(got2.cpu().numpy(), O.matmul_i8_f32(a[:, :256], q2, np.float32(0.02), m, 256, 768)) < 2e-5
    with pytest.raises(N.SbError):  # a view larger than the storage
        B200Backend.matmul_i8_f32(dev(a), b_q, np.float32(1.0), m, k, n + 1)
