"""The tensor-parallel decode pass (yskn_b200/tp_stack.py) and its pieces.

One GPU, each piece against the whole layer's call on the same inputs (bit for bit):
* a shard of several row ranges (yskn_b200_matrix_create_rows) gives the whole tensor's
  int64 sums of those rows, in range order;
* the Gated DeltaNet gates and step over each rank's run of value heads (the runs of the
  2-, 4- and 8-rank splits) give the whole layer's outputs, states and history for those
  heads and channels, over a committed row and a four-row call;
* the head merge of vocabulary parts gives the whole row's head_select (ties, NaN, -inf);
* the attention over a rank's query and KV heads at the one-GPU pass's fixed split count
  gives the whole launch's outputs for those heads.
Two GPUs (skipped with fewer): the whole tensor-parallel pass of a four-layer stack (three
Gated DeltaNet layers, one attention layer, small vocabulary) decodes the same tokens and
the same residual-stream bits as the one-GPU pass, token after token, eager and as a
CUDA graph.
"""
import os
import socket

import numpy as np
import pytest

import fixtures
import oracle as O

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def test_row_ranges_shard_is_the_whole_sums_of_those_rows(cuda):
    import torch
    import yskn_b200
    rows, cols = 3072, 2048
    words, lut16, sc16 = fixtures.model_matrix(rows, cols, 8, 31)
    si = O.signs("mulberry32_7919_13", 7, 0, cols)
    so = O.signs("mulberry32_7919_13", 7, cols, rows)
    dw = _dev(words.view(np.int32))
    whole = yskn_b200.Matrix(dw, "warp", rows, rows, cols, 8, lut16, sc16, si, so)
    M = 2
    rnd = fixtures.FixtureRandom(4)
    act = rnd.take(M * cols).astype(np.uint8).view(np.int8).reshape(M, cols).copy()
    A = (rnd.take(M * (cols // 512)) % 100000).astype(np.int32).reshape(M, -1)
    ref = torch.empty((M, rows), dtype=torch.int64, device="cuda")
    yskn_b200.weighted_sums([whole], _dev(act), _dev(A), [ref])
    ref = ref.cpu().numpy()
    for ranges in ([(0, 512), (1536, 2048), (2560, 3072)], [(2048, 3072), (512, 1024)], [(1024, 1536)]):
        m = yskn_b200.Matrix(dw, "warp", rows, rows, cols, 8, lut16, sc16, si, so, shard=(ranges, 0, cols))
        assert m.physical_rows == sum(b - a for a, b in ranges)
        out = torch.empty((M, m.physical_rows), dtype=torch.int64, device="cuda")
        yskn_b200.weighted_sums([m], _dev(act), _dev(A), [out])
        want = np.concatenate([ref[:, a:b] for a, b in ranges], axis=1)
        assert np.array_equal(out.cpu().numpy(), want), ranges
        # the fused operator restores each 512-row block with its own signs and scales
        x = fixtures.normal(8, cols).reshape(1, cols)
        work = torch.empty(yskn_b200.linear_work_bytes([m], 1), dtype=torch.uint8, device="cuda")
        y = torch.empty((1, m.rows), dtype=torch.float32, device="cuda")
        yskn_b200.linear([m], _dev(x), work, [y])
        work_w = torch.empty(yskn_b200.linear_work_bytes([whole], 1), dtype=torch.uint8, device="cuda")
        yw = torch.empty((1, rows), dtype=torch.float32, device="cuda")
        yskn_b200.linear([whole], _dev(x), work_w, [yw])
        yw = yw.cpu().numpy()
        assert np.array_equal(y.cpu().numpy().view(np.uint32),
                              np.concatenate([yw[:, a:b] for a, b in ranges], axis=1).view(np.uint32))
    assert yskn_b200.status() == 0


@pytest.mark.parametrize("mixer", [False, True])
def test_gdn_head_runs_equal_the_whole_layer(cuda, mixer):
    """Every rank's run of value heads (gates + step, or the one-launch mixer) gives the whole
    layer's outputs, states and history for those heads, for 2, 4 and 8 ranks."""
    import torch
    import yskn_b200
    from yskn_b200.tp_stack import TPPlan
    rng = np.random.default_rng(5)
    hidden, eps = 5120, 1e-6
    wb = O.bf16_bits((rng.standard_normal((48, hidden)) * 0.02).astype(np.float32))
    wa = O.bf16_bits((rng.standard_normal((48, hidden)) * 0.02).astype(np.float32))
    conv = O.bf16_bits((rng.standard_normal((10240, 4)) * 0.5).astype(np.float32))
    a_log = O.bf16_bits((rng.standard_normal(48) * 0.5).astype(np.float32))
    dt_bias = O.bf16_bits((rng.standard_normal(48) * 0.5).astype(np.float32))
    norm_w = O.bf16_bits((1 + rng.standard_normal(128) * 0.1).astype(np.float32))
    state0 = (rng.standard_normal((48, 128, 128)) * 0.1).astype(np.float32)
    hist0 = O.bf16_bits(rng.standard_normal((3, 10240)).astype(np.float32))
    calls = []
    for M, n_commit in [(1, 1), (4, 2)]:
        calls.append(dict(M=M, n_commit=n_commit,
                          x=O.bf16_bits(rng.standard_normal((M, hidden)).astype(np.float32)),
                          inv=(0.5 + rng.random(M)).astype(np.float32),
                          qkv=rng.standard_normal((M, 10240)).astype(np.float32),
                          z=rng.standard_normal((M, 6144)).astype(np.float32)))
    i16 = lambda a: _dev(a.view(np.int16))  # noqa: E731

    def run(v0, n_v, qk0, qk_ch, chans):
        """The run's outputs, gates, states and history over the calls (whole layer: None)."""
        whole = v0 is None
        hv = slice(0, 48) if whole else slice(v0, v0 + n_v)
        d_state = _dev(state0[hv])
        d_hist = i16(np.ascontiguousarray(hist0[:, chans]))
        res = []
        for c in calls:
            M = c["M"]
            nh = hv.stop - hv.start
            gates = torch.empty((M, 2 * nh), dtype=torch.float32, device="cuda")
            out = torch.empty((M, 128 * nh), dtype=torch.float32, device="cuda")
            if mixer and not whole:
                yskn_b200.gdn_mixer_heads(i16(c["x"]), _dev(c["inv"]), i16(np.ascontiguousarray(wb[hv])),
                                          i16(np.ascontiguousarray(wa[hv])),
                                          _dev(np.ascontiguousarray(c["qkv"][:, chans])),
                                          _dev(np.ascontiguousarray(c["z"][:, 128 * v0:128 * (v0 + n_v)])),
                                          i16(np.ascontiguousarray(conv[chans])), i16(np.ascontiguousarray(a_log[hv])),
                                          i16(np.ascontiguousarray(dt_bias[hv])), i16(norm_w), eps, d_state, d_hist,
                                          out, v0, qk0, qk_ch, n_commit=c["n_commit"])
                gates = None
            elif whole:
                yskn_b200.gdn_gates(i16(c["x"]), _dev(c["inv"]), i16(wb), i16(wa), gates)
                yskn_b200.gdn_step(_dev(c["qkv"]), _dev(c["z"]), gates, i16(conv), i16(a_log), i16(dt_bias),
                                   i16(norm_w), eps, d_state, d_hist, out, n_commit=c["n_commit"])
            else:
                yskn_b200.gdn_gates_heads(i16(c["x"]), _dev(c["inv"]), i16(np.ascontiguousarray(wb[hv])),
                                          i16(np.ascontiguousarray(wa[hv])), gates)
                yskn_b200.gdn_step_heads(_dev(np.ascontiguousarray(c["qkv"][:, chans])),
                                         _dev(np.ascontiguousarray(c["z"][:, 128 * v0:128 * (v0 + n_v)])), gates,
                                         i16(np.ascontiguousarray(conv[chans])), i16(np.ascontiguousarray(a_log[hv])),
                                         i16(np.ascontiguousarray(dt_bias[hv])), i16(norm_w), eps, d_state, d_hist,
                                         out, v0, qk0, qk_ch, n_commit=c["n_commit"])
            res.append((None if gates is None else gates.cpu().numpy(), out.cpu().numpy()))
        return res, d_state.cpu().numpy(), d_hist.cpu().numpy().view(np.uint16)

    ref, ref_state, ref_hist = run(None, None, None, None, np.arange(10240))
    for world in (2, 4, 8):
        for r in range(world):
            p = TPPlan(r, world)
            chans = np.concatenate([np.arange(a, b) for a, b in p.qkv_ranges])
            got, st, hist = run(p.v0, p.n_v, p.qk0, p.qk_ch, chans)
            hv = slice(p.v0, p.v0 + p.n_v)
            for (g, o), (rg, ro) in zip(got, ref):
                rgates = np.concatenate([rg[:, hv], rg[:, 48 + p.v0:48 + p.v0 + p.n_v]], axis=1)
                assert g is None or np.array_equal(g.view(np.uint32), rgates.view(np.uint32)), (world, r)
                assert np.array_equal(o.view(np.uint32), ro[:, 128 * p.v0:128 * (p.v0 + p.n_v)].view(np.uint32)), \
                    (world, r)
            assert np.array_equal(st.view(np.uint32), ref_state[hv].view(np.uint32)), (world, r)
            assert np.array_equal(hist, ref_hist[:, chans]), (world, r)
    assert yskn_b200.status() == 0


def test_head_merge_equals_the_whole_selection(cuda):
    import torch
    import yskn_b200
    rng = np.random.default_rng(9)
    n, M = 151936, 2
    logits = rng.standard_normal((M, n)).astype(np.float32)
    logits[0, [5, 70000, 151935]] = 9.0  # a three-way tie across parts: the smallest id wins
    logits[1, :1000] = np.nan
    logits[1, 1000:2000] = -np.inf
    logits[1, 140000] = 7.5
    d = _dev(logits)
    tok = torch.empty(M, dtype=torch.int32, device="cuda")
    tv = torch.empty((M, 8), dtype=torch.float32, device="cuda")
    ti = torch.empty((M, 8), dtype=torch.int32, device="cuda")
    yskn_b200.head_select(d, token=tok, top_logits=tv, top_ids=ti)
    from yskn_b200.tp import split_blocks
    for world in (2, 3, 8):
        ranges = split_blocks(n, world)
        pv = torch.empty((world, M, 8), dtype=torch.float32, device="cuda")
        pi = torch.empty((world, M, 8), dtype=torch.int32, device="cuda")
        for q, (a, b) in enumerate(ranges):
            yskn_b200.head_select(d[:, a:b].contiguous(), top_logits=pv[q], top_ids=pi[q])
        mt = torch.empty(M, dtype=torch.int32, device="cuda")
        mv = torch.empty((M, 8), dtype=torch.float32, device="cuda")
        mi = torch.empty((M, 8), dtype=torch.int32, device="cuda")
        yskn_b200.head_merge(pv, pi, [a for a, _ in ranges], token=mt, top_logits=mv, top_ids=mi)
        assert np.array_equal(mt.cpu().numpy(), tok.cpu().numpy()), world
        assert np.array_equal(mi.cpu().numpy(), ti.cpu().numpy()), world
        assert np.array_equal(mv.cpu().numpy().view(np.uint32), tv.cpu().numpy().view(np.uint32)), world
    assert tok.cpu().numpy()[0] == 5
    assert yskn_b200.status() == 0


def test_attention_on_a_ranks_heads_equals_the_whole_launch(cuda):
    import torch
    import yskn_b200
    from yskn_b200 import synthetic
    from yskn_b200.tp_stack import TPPlan
    n_qh, n_kvh, ctx = 24, 4, 700
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    cache = torch.randint(-2 ** 31, 2 ** 31, (2, n_kvh, ctx, 32), dtype=torch.int32, device="cuda", generator=g)
    scales = 0.02 + 0.18 * torch.rand((2, n_kvh, ctx), device="cuda", generator=g)
    rng = np.random.default_rng(2)
    q = _dev(O.bf16_bits(rng.standard_normal((1, n_qh, 256)).astype(np.float32)).view(np.int16))
    gate = _dev(O.bf16_bits(rng.standard_normal((1, n_qh, 256)).astype(np.float32)).view(np.int16))
    book = _dev(np.tile(synthetic.kv_codebook_bf16(), (n_kvh, 1)).view(np.int16))
    splits = 37

    def attend(qq, gg, c, s, nh):
        work = torch.empty(max(16, yskn_b200.kv4_attention_work_bytes(1, nh, ctx, splits)), dtype=torch.uint8,
                           device="cuda")
        out = torch.empty((1, nh, 256), dtype=torch.int16, device="cuda")
        yskn_b200.kv4_attention(qq, c[0], s[0], c[1], s[1], book[:c.shape[1]].contiguous(),
                                book[:c.shape[1]].contiguous(), ctx, work, out, gate=gg, n_splits=splits)
        return out.cpu().numpy()

    ref = attend(q, gate, cache, scales, n_qh)
    for world in (2, 4, 8):
        for r in range(world):
            p = TPPlan(r, world)
            hq = slice(p.h0, p.h0 + p.n_q)
            kv = slice(p.kv0, p.kv0 + p.n_kv)
            got = attend(q[:, hq].contiguous(), gate[:, hq].contiguous(), cache[:, kv].contiguous(),
                         scales[:, kv].contiguous(), p.n_q)
            assert np.array_equal(got, ref[:, hq]), (world, r)
    assert yskn_b200.status() == 0


_STACK = dict(layers=4, vocab=8192, ctx=96, bits=8, seed=3)
_TOKENS = 6


def _stack_tokens(st, stream, graph_tokens):
    """Eager tokens, then graph replays; the token and the residual stream after each."""
    import torch
    out = []
    for _ in range(_TOKENS):
        with torch.cuda.stream(stream):
            st.decode(stream)
        torch.cuda.synchronize()
        out.append((int(st.token.item()), st.h.cpu().numpy().copy()))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        st.decode(stream)
    for _ in range(graph_tokens):
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize()
        out.append((int(st.token.item()), st.h.cpu().numpy().copy()))
    del g
    return out


def _tp_stack_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    import yskn_b200
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from yskn_b200.tp_stack import TPStack
        st = TPStack(torch.device("cuda", rank), **_STACK)
        stream = torch.cuda.Stream()
        out = _stack_tokens(st, stream, 3)
        assert yskn_b200.status() == 0
        st.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_tp_stack_two_gpus_decodes_the_one_gpu_tokens(cuda):
    import torch
    import torch.multiprocessing as mp
    from yskn_b200 import stack as S
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    st = S.Stack(torch.device("cuda", 0), **_STACK)
    ref = _stack_tokens(st, torch.cuda.Stream(), 3)
    del st
    torch.cuda.empty_cache()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_stack_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert len({t for t, _ in ref}) > 1  # the tokens change from step to step
    for _, out in results:
        assert len(out) == len(ref)
        for k, ((t, h), (rt, rh)) in enumerate(zip(out, ref)):
            assert t == rt, k
            assert np.array_equal(h.view(np.uint16), rh.view(np.uint16)), k
