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


def _case(seed, B=3, n_q=32, n_kv=8, hd=128, page=16, lens=(1, 37, 300)):
    rng = np.random.default_rng(seed)
    max_pages = (max(lens) + page - 1) // page
    perm = rng.permutation(B * max_pages)
    kp = np.zeros((B * max_pages, n_kv, page, hd), np.float32)
    vp = np.zeros_like(kp)
    tables = np.zeros((B, max_pages), np.int32)
    for b, S in enumerate(lens):
        k = O.round_bf16(rng.standard_normal((S, n_kv * hd)).astype(np.float32))
        v = O.round_bf16(rng.standard_normal((S, n_kv * hd)).astype(np.float32))
        for i in range((S + page - 1) // page):
            pg = perm[b * max_pages + i]
            tables[b, i] = pg
            kp[pg, :, : min(page, S - i * page)] = k[i * page:(i + 1) * page].reshape(-1, n_kv, hd).transpose(1, 0, 2)
            vp[pg, :, : min(page, S - i * page)] = v[i * page:(i + 1) * page].reshape(-1, n_kv, hd).transpose(1, 0, 2)
    q = (rng.standard_normal((B, n_q * hd)) / np.sqrt(hd)).astype(np.float32)
    d = dict(q=torch.from_numpy(q).cuda(), k=torch.from_numpy(kp).cuda().to(torch.bfloat16),
             v=torch.from_numpy(vp).cuda().to(torch.bfloat16), t=torch.from_numpy(tables).cuda(),
             l=torch.tensor(list(lens), dtype=torch.int32).cuda())
    return d, dict(B=B, n_q=n_q, n_kv=n_kv, hd=hd, page=page, max_pages=max_pages)


def _call(fn, d, s, out):
    return fn(_vp(d["q"]), _vp(d["k"]), _vp(d["v"]), N.SB_KV_BF16, _vp(d["t"]), s["max_pages"], _vp(d["l"]), s["B"],
              s["n_q"], s["n_kv"], s["hd"], s["page"], s["max_pages"] * s["page"], _vp(out), None)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    N.check(N.lib().sb_init(0))
    d, s = _case(11)
    ref = torch.empty_like(d["q"])
    N.check(_call(N.lib().sb_attn_decode_paged, d, s, ref))
    torch.cuda.synchronize()
    for _ in range(2):  # the fixed scratch keeps the previous call's contents
        out = torch.full_like(d["q"], float("nan"))
        N.check(_call(N.lib().sb_attn_decode_paged_noalloc, d, s, out))
        torch.cuda.synchronize()
        assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5


def test_noalloc_rejects_shapes_beyond_its_scratch():
    N.check(N.lib().sb_init(0))
    # 4 sequences x 64 query heads x 10 splits x 130 floats = 1.33 MB > 1 MiB of partials
    d, s = _case(12, B=4, n_q=64, n_kv=8, hd=128, page=16, lens=(300, 300, 300, 300))
    out = torch.empty_like(d["q"])
    rc = _call(N.lib().sb_attn_decode_paged_noalloc, d, s, out)
    assert rc == 4 and "fixed scratch" in N.last_error()
