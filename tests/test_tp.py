"""Tensor parallelism: weight sharding (host), the row/column-split algebra
over gloo ranks on the CPU, and the NCCL tensor-parallel engine on 2 GPUs.

The reference runs on one device, so its oracle for the sharded path is the
unsharded model: a TP engine must hold slices of exactly the reference int8
tensors (full-tensor scales), and greedy streams must equal the oracle's.
"""
import os
import socket

import numpy as np
import pytest

import oracle as O
from esolearn_b200 import LlamaConfig, QuantLlamaB200, tp_shard_qweight, tp_shard_shape
from esolearn_b200 import _native as N

from gpu_util import engine_from_oracle, orc_config, rel_err, small_config


def _cfg(T=1):
    # GQA 8 query / 4 kv heads, hd 32, ffn 96, vocab 64; for 8 ranks 16 query /
    # 8 kv heads of 16
    if T == 8:
        return LlamaConfig(64, 256, 96, 2, 16, 8, 128, 1e-5, 10000.0, False, None)
    return LlamaConfig(64, 256, 96, 2, 8, 4, 128, 1e-5, 10000.0, False, None)


@pytest.mark.parametrize("T", [1, 2, 4, 8])
def test_shards_partition_every_weight(T):
    c = _cfg(T)
    hd = c.head_dim()
    Qf, KVf = c.n_heads * hd, c.n_kv_heads * hd
    rng = np.random.default_rng(T)
    full = {
        N.SB_W_QKV: rng.integers(-127, 128, (c.hidden_size, Qf + 2 * KVf), dtype=np.int8),
        N.SB_W_O: rng.integers(-127, 128, (Qf, c.hidden_size), dtype=np.int8),
        N.SB_W_GATE: rng.integers(-127, 128, (c.hidden_size, c.intermediate_size), dtype=np.int8),
        N.SB_W_UP: rng.integers(-127, 128, (c.hidden_size, c.intermediate_size), dtype=np.int8),
        N.SB_W_DOWN: rng.integers(-127, 128, (c.intermediate_size, c.hidden_size), dtype=np.int8),
        N.SB_W_LM_HEAD: rng.integers(-127, 128, (c.vocab_size, c.hidden_size), dtype=np.int8),
    }
    for slot, w in full.items():
        parts = [tp_shard_qweight(c, slot, r, T, w) for r in range(T)]
        for r, p in enumerate(parts):
            assert p.shape == tp_shard_shape(c, slot, r, T)
        if slot == N.SB_W_QKV:
            q, k, v = Qf // T, KVf // T, KVf // T
            re = np.concatenate([np.concatenate([p[:, :q] for p in parts], 1),
                                 np.concatenate([p[:, q:q + k] for p in parts], 1),
                                 np.concatenate([p[:, q + k:] for p in parts], 1)], 1)
        elif slot in (N.SB_W_GATE, N.SB_W_UP):
            re = np.concatenate(parts, 1)
        else:  # o, down, lm_head: row slices
            re = np.concatenate(parts, 0)
        assert np.array_equal(re, w), slot


def test_shard_rejects_uneven_splits():
    c = _cfg()
    with pytest.raises(N.SbError) as ei:
        tp_shard_shape(c, N.SB_W_O, 0, 3)
    assert ei.value.code == 4  # SB_ERR_SHAPE
    with pytest.raises(N.SbError):
        tp_shard_shape(c, N.SB_W_O, 2, 2)  # rank out of range


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gloo_worker(rank, size, port, out):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        c = _cfg()
        rng = np.random.default_rng(7)
        M = 3
        hd = c.head_dim()
        Qf = c.n_heads * hd
        wo = (rng.standard_normal((Qf, c.hidden_size)) * 0.02).astype(np.float32)
        wg = (rng.standard_normal((c.hidden_size, c.intermediate_size)) * 0.02).astype(np.float32)
        qo, so = O.quantize_symmetric(wo)
        qg, sg = O.quantize_symmetric(wg)
        qo, qg = qo.reshape(wo.shape), qg.reshape(wg.shape)
        a_attn = rng.standard_normal((M, Qf)).astype(np.float32)
        a_x = rng.standard_normal((M, c.hidden_size)).astype(np.float32)
        # o: row split (this rank's heads of the attention output), partial sums all-reduced
        po = tp_shard_qweight(c, N.SB_W_O, rank, size, qo)
        rows = po.shape[0]
        part = O.matmul_i8_f32(np.ascontiguousarray(a_attn[:, rank * rows:(rank + 1) * rows]), po, so, M, rows,
                               c.hidden_size)
        t = torch.from_numpy(np.ascontiguousarray(part))
        dist.all_reduce(t)
        full_o = O.matmul_i8_f32(a_attn, qo, so, M, Qf, c.hidden_size)
        # gate: column split, gathered
        pg = tp_shard_qweight(c, N.SB_W_GATE, rank, size, qg)
        yg = torch.from_numpy(O.matmul_i8_f32(a_x, pg, sg, M, c.hidden_size, pg.shape[1]))
        gathered = [torch.empty_like(yg) for _ in range(size)]
        dist.all_gather(gathered, yg)
        full_g = O.matmul_i8_f32(a_x, qg, sg, M, c.hidden_size, c.intermediate_size)
        if rank == 0:
            out.put((rel_err(t.numpy(), full_o), bool(np.array_equal(torch.cat(gathered, 1).numpy(), full_g))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("size", [2, 4])
def test_row_and_column_splits_over_gloo_ranks(size):
    # World size 2 or 4 on the CPU: the o projection's row split summed by an
    # all-reduce equals the unsharded product within f32 rounding, and the
    # gate projection's column split gathered equals it bit for bit.
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, size, port, q)) for r in range(size)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    err, col_equal = q.get(timeout=10)
    assert err < 1e-6, err
    assert col_equal


# ---------------------------------------------------------------------------
# the NCCL tensor-parallel engine on 2 GPUs

def _tp_config(size=2):
    # GQA 8 query / 4 kv heads, head_dim 64; 16 / 8 heads for 8 ranks (one kv head each)
    if size > 4:
        return small_config(h=1024, layers=2, heads=16, kv=8, ffn=1024, vocab=1024)
    return small_config(h=512, layers=2, heads=8, kv=4, ffn=512, vocab=1024)


def _tp_engine_worker(rank, size, tid, mode, out):
    try:
        out.put(_tp_engine_run(rank, size, tid, mode))
    except BaseException:  # report instead of leaving the parent waiting
        import traceback

        out.put((rank, "error", traceback.format_exc(), None))


VARYING_BATCHES = (64, 8, 64, 8, 1, 64, 1, 1, 64)


def _varying_config():
    # hidden 4096: every batched all-reduce of M >= 8 rows carries M*h >= 32768 values
    return small_config(h=4096, layers=1, heads=32, kv=8, ffn=512, vocab=1024)


def _varying_tokens(i, M):
    return O.prompt_ids(500 + i, M, _varying_config().vocab_size)


def _tp_engine_run(rank, size, tid, mode):
    import torch

    torch.cuda.set_device(rank)
    N.check(N.lib().sb_init(rank))
    if mode == "varying":
        # The batch size changes from step to step (64, 8, 1 rows), so the
        # residual all-reduces alternate between large and small vectors; a
        # cell left by an earlier all-reduce must never pass for this one's.
        c = _varying_config()
        om = O.OracleLlama(orc_config(c, 64), 6)
        e = engine_from_oracle(om, c, max_seq=64, max_batch=64, kv_dtype="bf16", tp_rank=rank, tp_size=size,
                               tp_id=tid)
        outs = []
        for i, M in enumerate(VARYING_BATCHES):
            lg, _ = e.forward_batch(_varying_tokens(i, M).tolist(), [0] * M)
            outs.append(lg)
        e.close()
        return rank, outs, None, None
    if mode == "oracle":
        c = _tp_config(size)
        om = O.OracleLlama(orc_config(c, 128), 5)
        e = engine_from_oracle(om, c, max_seq=128, max_batch=4, kv_dtype="bf16", tp_rank=rank, tp_size=size,
                               tp_id=tid)
    else:  # on-device random init, checked shard by shard against the oracle's generator
        c = _tp_config(size)
        e = QuantLlamaB200.new_random(c, 3, max_seq=128, max_batch=4, kv_dtype="bf16", tp_rank=rank, tp_size=size,
                                      tp_id=tid)
        om = O.OracleLlama(orc_config(c, 128), 3)
        for l in range(c.n_layers):
            for slot in range(5):
                qg, sg = e.get_qweight(l, slot)
                qo, so = om.weight(l, slot)
                assert sg == so and np.array_equal(qg, tp_shard_qweight(c, slot, rank, size, qo)), (l, slot)
        qg, sg = e.get_qweight(-1, 0)
        qo, so = om.lm_head()
        assert sg == so and np.array_equal(qg, tp_shard_qweight(c, N.SB_W_LM_HEAD, rank, size, qo))
    prompt = O.prompt_ids(11, 8, c.vocab_size)
    toks1 = e.generate_greedy(prompt, 32)[0]
    prompts = np.stack([O.prompt_ids(20 + b, 8, c.vocab_size) for b in range(3)])
    toks3 = e.generate_greedy(prompts, 32)
    cache = e.new_kv_cache(64)
    lg = np.stack([e.forward_with_cache(int(t), pos, cache) for pos, t in enumerate(prompt)])
    e.close()
    return rank, toks1, toks3, lg


@pytest.mark.gpu
@pytest.mark.parametrize("size", [2, 4, 8])
@pytest.mark.parametrize("mode", ["oracle", "random"])
def test_tensor_parallel_engine_matches_oracle(mode, size):
    # 2, 4 or 8 ranks (NCCL over NVLink, peer-memory exchanges): greedy
    # streams for 1 sequence (the persistent step, exchanging inside the
    # kernel) and 3 sequences (per-operation kernels) equal the unsharded
    # oracle's for 32 tokens, logits within the f32 bar, on every rank.
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < size:
        pytest.skip(f"needs {size} GPUs")
    from esolearn_b200 import tp_unique_id

    tid = tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_engine_worker, args=(r, size, tid, mode, q), daemon=True) for r in range(size)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(size):
            r, t1, t3, lg = q.get(timeout=300)
            assert not (isinstance(t1, str) and t1 == "error"), f"rank {r}:\n{t3}"
            res[r] = (t1, t3, lg)
        for p in procs:
            p.join(60)
            assert p.exitcode == 0
    finally:
        for p in procs:  # a rank left waiting on a failed peer ends with the test
            if p.is_alive():
                p.kill()
    c = _tp_config(size)
    om = O.OracleLlama(orc_config(c, 128), 5 if mode == "oracle" else 3)
    prompt = O.prompt_ids(11, 8, c.vocab_size)
    ref1 = om.generate_greedy(prompt, 32, kv_bf16=True)
    oc = om.new_cache(64, kv_bf16=True)
    ref_lg = np.stack([om.forward_with_cache(oc, int(t), pos) for pos, t in enumerate(prompt)])
    for r in range(size):
        t1, t3, lg = res[r]
        assert t1.tolist() == ref1.tolist(), r
        for b in range(3):
            assert t3[b].tolist() == om.generate_greedy(O.prompt_ids(20 + b, 8, c.vocab_size), 32,
                                                        kv_bf16=True).tolist(), (r, b)
        assert rel_err(lg, ref_lg) < 1e-3
    for r in range(1, size):
        assert np.array_equal(res[0][2], res[r][2])  # identical logits on every rank


@pytest.mark.gpu
def test_tensor_parallel_batch_size_changes_between_steps():
    # 2 ranks; consecutive steps of 64, 8 and 1 rows (h 4096): every row's
    # logits equal the unsharded oracle's (fresh sequence, position 0) within
    # the f32 bar on both ranks, with identical bits on the two ranks.
    import torch
    import torch.multiprocessing as mp

    size = 2
    if torch.cuda.device_count() < size:
        pytest.skip(f"needs {size} GPUs")
    from esolearn_b200 import tp_unique_id

    tid = tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_engine_worker, args=(r, size, tid, "varying", q), daemon=True)
             for r in range(size)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(size):
            r, outs, err, _ = q.get(timeout=300)
            assert not (isinstance(outs, str) and outs == "error"), f"rank {r}:\n{err}"
            res[r] = outs
        for p in procs:
            p.join(60)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    c = _varying_config()
    om = O.OracleLlama(orc_config(c, 64), 6)
    memo = {}
    for i, M in enumerate(VARYING_BATCHES):
        for b, t in enumerate(_varying_tokens(i, M).tolist()):
            if t not in memo:
                memo[t] = om.forward_with_cache(om.new_cache(4, kv_bf16=True), t, 0)
            assert rel_err(res[0][i][b], memo[t]) < 1e-3, (i, M, b)
            assert np.array_equal(res[0][i][b], res[1][i][b]), (i, M, b)


@pytest.mark.gpu
def test_peer_allreduce_wait_gives_up_and_device_stays_usable():
    # A rank that never delivers its partial sums: the peer all-reduce's
    # bounded wait (2 s of %globaltimer) raises its error word instead of
    # hanging, and the device keeps working afterwards.
    import ctypes as C

    import torch

    from esolearn_b200 import QWeight, matmul_i8_f32

    N.check(N.lib().sb_init(0))
    timed_out, secs = C.c_int32(0), C.c_double(0)
    N.check(N.lib().sb_tp_probe_timeout(C.byref(timed_out), C.byref(secs)))
    assert timed_out.value == 1
    assert 1.5 < secs.value < 30.0, secs.value
    rng = np.random.default_rng(0)
    q = rng.integers(-127, 128, (64, 32), dtype=np.int8)
    a = rng.standard_normal((2, 64)).astype(np.float32)
    out = matmul_i8_f32(torch.from_numpy(a).cuda(), QWeight(q, [0.01])).cpu().numpy()
    assert rel_err(out, O.matmul_i8_f32(a, q, np.float32(0.01), 2, 64, 32)) < 1e-5
