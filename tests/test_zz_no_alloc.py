"""The allocation-free attention entry point (sb_attn_decode_paged_noalloc).

It serves callers that cannot let the library allocate device memory (their
own pool owns all of it, or an allocation's synchronisation is unaffordable
mid-step), so it keeps its split scratch in a fixed array inside the
library.  This file is collected last so that a failure here comes after
every other test has run; it must pass alone and after the other tests.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from esolearn_b200 import _native as N
from tests.gpu_util import rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _vp(t):
    return C.c_void_p(t.data_ptr())


def _splits(B, n_kv, max_ctx):
    """Context splits both entry points choose (attn_pick_splits, attention.cu):
    two waves of CTAs over the device's SMs, at most about 256 positions per
    split, at least 16 positions per split, 1..64."""
    sms = C.c_int32()
    N.check(N.lib().sb_device_info(C.byref(sms), None, None, None))
    s = max(-(-2 * sms.value // (B * n_kv)), -(-max_ctx // 256))
    s = min(s, -(-max_ctx // 16))
    return max(1, min(s, 64))


def _case(seed, B=3, n_q=32, n_kv=8, hd=128, page=16, lens=(1, 37, 300)):
    rng = np.random.default_rng(seed)
    refs = []
    max_pages = (max(lens) + page - 1) // page
    perm = rng.permutation(B * max_pages)
    kp = np.zeros((B * max_pages, n_kv, page, hd), np.float32)
    vp = np.zeros_like(kp)
    tables = np.zeros((B, max_pages), np.int32)
    for b, S in enumerate(lens):
        k = O.round_bf16(rng.standard_normal((S, n_kv * hd)).astype(np.float32))
        v = O.round_bf16(rng.standard_normal((S, n_kv * hd)).astype(np.float32))
        refs.append((k, v))
        for i in range((S + page - 1) // page):
            pg = perm[b * max_pages + i]
            tables[b, i] = pg
            kp[pg, :, : min(page, S - i * page)] = k[i * page:(i + 1) * page].reshape(-1, n_kv, hd).transpose(1, 0, 2)
            vp[pg, :, : min(page, S - i * page)] = v[i * page:(i + 1) * page].reshape(-1, n_kv, hd).transpose(1, 0, 2)
    q = (rng.standard_normal((B, n_q * hd)) / np.sqrt(hd)).astype(np.float32)
    d = dict(q=torch.from_numpy(q).cuda(), k=torch.from_numpy(kp).cuda().to(torch.bfloat16),
             v=torch.from_numpy(vp).cuda().to(torch.bfloat16), t=torch.from_numpy(tables).cuda(),
             l=torch.tensor(list(lens), dtype=torch.int32).cuda())
    # the reference decode attention (llama.rs:414-456) of each sequence
    d["ref"] = np.stack([O.attention_decode(q[b], k, v, n_q, n_kv, hd) for b, (k, v) in enumerate(refs)])
    return d, dict(B=B, n_q=n_q, n_kv=n_kv, hd=hd, page=page, max_pages=max_pages)


def _call(fn, d, s, out):
    return fn(_vp(d["q"]), _vp(d["k"]), _vp(d["v"]), N.SB_KV_BF16, _vp(d["t"]), s["max_pages"], _vp(d["l"]), s["B"],
              s["n_q"], s["n_kv"], s["hd"], s["page"], s["max_pages"] * s["page"], _vp(out), None)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    N.check(N.lib().sb_init(0))
    d, s = _case(11)
    # the split path (partials and counters in the fixed scratch) must run
    assert _splits(s["B"], s["n_kv"], s["max_pages"] * s["page"]) > 1
    ref = torch.empty_like(d["q"])
    N.check(_call(N.lib().sb_attn_decode_paged, d, s, ref))
    torch.cuda.synchronize()
    ref = ref.cpu().numpy()
    for b in range(s["B"]):
        assert rel_err(ref[b], d["ref"][b]) < 1e-5, b
    for _ in range(2):  # the fixed scratch keeps the previous call's contents
        out = torch.full_like(d["q"], float("nan"))
        N.check(_call(N.lib().sb_attn_decode_paged_noalloc, d, s, out))
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert rel_err(got, ref) < 1e-5
        for b in range(s["B"]):
            assert rel_err(got[b], d["ref"][b]) < 1e-5, b


def test_noalloc_rejects_shapes_beyond_its_scratch():
    N.check(N.lib().sb_init(0))
    # 4 sequences x 64 query heads x 10 splits (148 SMs) x 130 floats = 1.33 MB > 1 MiB of partials
    d, s = _case(12, B=4, n_q=64, n_kv=8, hd=128, page=16, lens=(300, 300, 300, 300))
    splits = _splits(s["B"], s["n_kv"], s["max_pages"] * s["page"])
    assert 4 * s["B"] * s["n_q"] * splits * (s["hd"] + 2) > 1024 * 1024, splits
    out = torch.empty_like(d["q"])
    rc = _call(N.lib().sb_attn_decode_paged_noalloc, d, s, out)
    assert rc == 4 and "fixed scratch" in N.last_error()
