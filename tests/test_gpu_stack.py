"""The decode pass of the 27B-shape hybrid stack (yskn_b200/stack.py) on a short stack:
four layers (three Gated DeltaNet, one attention), a 4,096-row head and a 256-row KV cache.
Every call reports success, the greedy token stays inside the vocabulary, and the pass
captured as a CUDA graph produces the same tokens, hidden rows and recurrent states, bit
for bit, as the same pass run eagerly from the same starting state."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def test_stack_graph_equals_eager(cuda):
    import torch
    import yskn_b200 as Y
    from yskn_b200 import stack as S

    def run(use_graph, tokens=3):
        st = S.Stack(cuda, layers=4, vocab=4096, ctx=256, seed=5)
        stream = torch.cuda.Stream(cuda)
        out = []
        if use_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                st.decode(stream)  # set-up outside capture (this is the first token)
            torch.cuda.synchronize()
            out.append(int(st.token.item()))
            with torch.cuda.graph(graph, stream=stream):
                st.decode(stream)
            # capture does not run the pass: states are as after the first token
            for _ in range(tokens - 1):
                with torch.cuda.stream(stream):
                    graph.replay()
                torch.cuda.synchronize()
                out.append(int(st.token.item()))
        else:
            for _ in range(tokens):
                with torch.cuda.stream(stream):
                    st.decode(stream)
                torch.cuda.synchronize()
                out.append(int(st.token.item()))
        assert Y.status(stream) == 0
        return out, st.h.clone(), [L["state"].clone() for L in st.L if L["kind"] == "gdn"], st.logits.clone()

    a_tok, a_h, a_states, a_logits = run(False)
    b_tok, b_h, b_states, b_logits = run(True)
    assert all(0 <= t < 4096 for t in a_tok)
    assert a_tok == b_tok
    assert torch.equal(a_h, b_h)
    assert torch.equal(a_logits.view(torch.int32), b_logits.view(torch.int32))
    for x, y in zip(a_states, b_states):
        assert torch.equal(x.view(torch.int32), y.view(torch.int32))
    assert torch.isfinite(a_logits).all()


# ------------------------------------------------------------------------------------------
# The stack against the composed oracle: one Gated DeltaNet layer and one attention layer.

def _host_u32(t):
    return t.cpu().numpy().view(np.uint32)


def _host_u16(t):
    return t.cpu().numpy().view(np.uint16)


def _kv_profile():
    """The stack's KV profile (tables (s*73+19)%2049-1024 with gain 257/256, multipliers
    0.9/1.0/1.1, 4-bit groups) as the oracle encoder reads it."""
    import struct
    import kv
    b = kv.test_profile(1, 4, 4)
    to = struct.unpack_from("<I", b, 112)[0]
    struct.pack_into("<f", b, to + 4, 257.0 / 256.0)
    return kv.parse_profile(b)


class _OracleStack:
    """The oracle's own decode pass over the weights of a yskn_b200.stack.Stack: every step
    is an oracle function (oracle/oracle.py, oracle/kv.py), composed in the order of
    Stack.decode; nothing of the device's intermediate values is used."""

    def __init__(self, st):
        import kv
        self.st, self.kv = st, kv
        self.rule = "mulberry32_7919_13"
        self.book = __import__("yskn_b200.synthetic", fromlist=["kv_codebook_bf16"]).kv_codebook_bf16()
        self.profile = _kv_profile()
        self.L = []
        for L in st.L:
            H = {"kind": L["kind"], "in_norm": _host_u16(L["in_norm"]), "post_norm": _host_u16(L["post_norm"])}
            for k, v in L.items():
                if hasattr(v, "source"):
                    H[k] = self._spec(v)
            if L["kind"] == "gdn":
                for k in ("wb", "wa", "conv", "a_log", "dt_bias", "norm_w"):
                    H[k] = _host_u16(L[k])
                H["state"] = L["state"].cpu().numpy().copy()
                H["history"] = _host_u16(L["history"]).copy()
            else:
                H["q_norm"], H["k_norm"] = _host_u16(L["q_norm"]), _host_u16(L["k_norm"])
                H["cache"] = _host_u32(L["cache"]).copy()
                H["scales"] = L["scales"].cpu().numpy().copy()
            self.L.append(H)
        self.final_norm = _host_u16(st.final_norm)
        self.head = self._spec(st.head)
        w, lut, sc = st.embedding_source
        self.emb = [(_host_u32(w), "row", st.vocab, 5120, st.bits, np.asarray(lut), np.asarray(sc))]

    def _spec(self, m):
        words, lut16, sc16, rotate = m.source
        rows, cols = m.physical_rows, m.cols
        si = O.signs(self.rule, 7, 0, cols)
        so = O.signs(self.rule, 7, cols, rows) if rotate else None
        return (_host_u32(words), rows, cols, np.asarray(lut16), np.asarray(sc16), si, so)

    def lin(self, spec, x, inv=None):
        words, rows, cols, lut16, sc16, si, so = spec
        lut8, tau = O.quantize_weight_table(lut16, sc16)
        act8, _, A, rq = O.quantize_activation(np.asarray(x, np.float32).reshape(1, cols), si)
        ws = O.fast_weighted_sums(words, "warp", rows, cols, self.st.bits, lut8, act8, A)
        return O.restore(ws, rq, tau, so, None if inv is None else np.array([inv], np.float32))[0]

    def attention(self, H, x, inv):
        kv, ctx = self.kv, self.st.ctx
        q = self.lin(H["q"], x, inv).reshape(24, 512)
        k = self.lin(H["k"], x, inv).reshape(4, 256)
        v = self.lin(H["v"], x, inv).reshape(4, 256)
        query, gate, kr, vr = O.attention_prep(q, k, v, H["q_norm"], H["k_norm"], ctx, 1e-6)
        for side, rows in ((0, kr), (1, vr)):
            for h in range(4):
                kind, scale, words, *_ = kv.encode(self.profile, 2 * h + side, ctx, rows[h])
                assert kind == 4
                H["cache"][side, h, ctx] = words
                H["scales"][side, h, ctx] = scale
        n = ctx + 1
        splits = 31 if n < 4096 else 42  # attention.rs:207-232
        out = np.empty((24, 256), np.float32)
        for j in range(24):
            h = j // 6
            kb = kv.decode_packed_rows(H["cache"][0, h, :n], 4, self.book)
            vb = kv.decode_packed_rows(H["cache"][1, h, :n], 4, self.book)
            att = kv.attend_head(O.bf16_float(query[j]), kb, H["scales"][0, h, :n], vb, H["scales"][1, h, :n],
                                 np.zeros(256, np.float32), n, splits)  # packed rows add +0 * den (attention.rs:354-366)
            r = O.bf16_float(O.bf16_bits(kv.inverse_rotate(att)))
            sg = O.bf16_float(O.bf16_bits(O.pm("sigmoid", O.bf16_float(gate[j]))))
            out[j] = O.bf16_float(O.bf16_bits(r * sg))
        return out

    def tail(self, H, h, a_out):
        """o_proj of a given attention output, then the layer's MLP: (hidden, proj)."""
        proj = self.lin(H["o"], a_out.reshape(-1))
        return self.mlp(H, h, proj)

    def mlp(self, H, h, proj):
        h, x, inv, _ = O.residual_prepare(h, proj, H["post_norm"], 1e-6)
        g, u = self.lin(H["gate"], x, inv), self.lin(H["up"], x, inv)
        return h, self.lin(H["down"], O.gated_product(g, u))

    def token(self, tok):
        """One decode step from token `tok`: (greedy token, logits, hidden bits, per layer
        the attention output or None)."""
        h = O.embedding_rows(self.emb, [tok], O.signs(self.rule, 7, 0, 5120))[0]
        proj, att_out = None, []
        for H in self.L:
            h, x, inv, xg = O.residual_prepare(h, proj, H["in_norm"], 1e-6)
            if H["kind"] == "gdn":
                qkv, z = self.lin(H["qkv"], x, inv), self.lin(H["z"], x, inv)
                gates = O.gdn_gates(xg, inv, H["wb"], H["wa"])
                out, H["state"], H["history"] = O.gdn_step(qkv[None], z[None], gates[None], H["conv"], H["a_log"],
                                                           H["dt_bias"], H["norm_w"], 1e-6, H["state"], H["history"])
                h, proj = self.mlp(H, h, self.lin(H["out"], out[0]))
                att_out.append(None)
            else:
                a = self.attention(H, x, inv)
                att_out.append(a)
                h, proj = self.tail(H, h, a)
        h, x, inv, _ = O.residual_prepare(h, proj, self.final_norm, 1e-6)
        logits = self.lin(self.head, x, inv)
        return O.head_select(logits)[0], logits, h, att_out


def test_two_layer_stack_matches_the_composed_oracle(cuda):
    """One Gated DeltaNet layer then one attention layer (hidden 5120, the 27B layer shapes,
    a 1,024-row head, a 64-row KV cache), two tokens, against the oracle's own pass from the
    same weights and inputs:
    * through the GDN layer and up to the attention everything is bit-exact: the hidden row
      after layer 0, the recurrent state and convolution history, the encoded KV rows;
    * the attention output (bf16, after the inverse rotation and the gate) lies within the
      attention tolerance of tests/test_gpu_kv.py: |gpu - oracle| <= 2^-7 |oracle| +
      8e-3 max |oracle| (the spec leaves the MMA order open, ATT-01);
    * given the device's attention output, the rest of the pass (o_proj, residual, MLP,
      final norm, head logits, greedy token) is bit-exact;
    * the oracle's independent logits lie within 5e-2 of the largest logit of the device's."""
    import torch
    import yskn_b200 as Y
    from yskn_b200 import stack as S
    st = S.Stack(cuda, vocab=1024, ctx=64, seed=9, kinds=["gdn", "attn"])
    orc = _OracleStack(st)
    stream = torch.cuda.Stream(cuda)
    tok = 17
    for step in range(2):
        st.token.fill_(tok)
        with torch.cuda.stream(stream):
            st.decode(stream)
        torch.cuda.synchronize()
        assert Y.status(stream) == 0
        o_tok, o_logits, o_h, o_att = orc.token(tok)
        # Layer 0 (GDN) state and history: bit-exact.
        g = st.L[0]
        assert np.array_equal(g["state"].cpu().numpy().view(np.uint32), orc.L[0]["state"].view(np.uint32)), step
        assert np.array_equal(_host_u16(g["history"]), orc.L[0]["history"]), step
        # The encoded KV rows of this token: bit-exact words and scales.
        a = st.L[1]
        assert np.array_equal(_host_u32(a["cache"])[:, :, st.ctx], orc.L[1]["cache"][:, :, st.ctx]), step
        assert np.array_equal(a["scales"].cpu().numpy()[:, :, st.ctx].view(np.uint32),
                              orc.L[1]["scales"][:, :, st.ctx].view(np.uint32)), step
        # The attention output within the attention tolerance.
        dev_att = O.bf16_float(_host_u16(st.a_out)[0])
        want = o_att[1]
        assert np.all(np.abs(dev_att - want) <= 2.0 ** -7 * np.abs(want) + 8e-3 * np.abs(want).max()), step
        # Independent logits within tolerance.
        dev_logits = st.logits.cpu().numpy()[0]
        assert np.abs(dev_logits - o_logits).max() <= 5e-2 * np.abs(dev_logits).max(), step
        tok = int(st.token.item())
        assert 0 <= tok < 1024
    # The rest of the pass given the device's attention output, on a fresh pair (one token).
    st2 = S.Stack(cuda, vocab=1024, ctx=64, seed=9, kinds=["gdn", "attn"])
    orc2 = _OracleStack(st2)
    st2.token.fill_(5)
    with torch.cuda.stream(stream):
        st2.decode(stream)
    torch.cuda.synchronize()
    h = O.embedding_rows(orc2.emb, [5], O.signs(orc2.rule, 7, 0, 5120))[0]
    H0, H1 = orc2.L
    h, x, inv, xg = O.residual_prepare(h, None, H0["in_norm"], 1e-6)
    qkv, z = orc2.lin(H0["qkv"], x, inv), orc2.lin(H0["z"], x, inv)
    gates = O.gdn_gates(xg, inv, H0["wb"], H0["wa"])
    out, _, _ = O.gdn_step(qkv[None], z[None], gates[None], H0["conv"], H0["a_log"], H0["dt_bias"], H0["norm_w"],
                           1e-6, H0["state"], H0["history"])
    h, proj = orc2.mlp(H0, h, orc2.lin(H0["out"], out[0]))
    h, x, inv, _ = O.residual_prepare(h, proj, H1["in_norm"], 1e-6)
    dev_att = O.bf16_float(_host_u16(st2.a_out)[0])
    h, proj = orc2.tail(H1, h, dev_att)
    h, x, inv, _ = O.residual_prepare(h, proj, orc2.final_norm, 1e-6)
    logits = orc2.lin(orc2.head, x, inv)
    assert np.array_equal(_host_u16(st2.h)[0], h)
    assert np.array_equal(st2.logits.cpu().numpy()[0].view(np.uint32), logits.view(np.uint32))
    assert int(st2.token.item()) == O.head_select(logits)[0]


def test_fused_chain_pass_equals_the_separate_calls(cuda):
    """The decode pass with the chain between projections inside the operators (436 launches
    per token) and with the separate residual/normalisation and product calls (660): the
    same tokens, hidden rows, logits and recurrent states, bit for bit, over three tokens."""
    import torch
    import yskn_b200 as Y
    from yskn_b200 import stack as S

    def run(fused):
        st = S.Stack(cuda, layers=4, vocab=4096, ctx=128, seed=13)
        stream = torch.cuda.Stream(cuda)
        toks = []
        for _ in range(3):
            with torch.cuda.stream(stream):
                st.decode(stream, fused=fused)
            torch.cuda.synchronize()
            toks.append(int(st.token.item()))
        assert Y.status(stream) == 0
        return toks, st.h.clone(), st.logits.clone(), [L["state"].clone() for L in st.L if L["kind"] == "gdn"]

    a = run(True)
    b = run(False)
    assert a[0] == b[0]
    assert torch.equal(a[1], b[1])
    assert torch.equal(a[2].view(torch.int32), b[2].view(torch.int32))
    for x, y in zip(a[3], b[3]):
        assert torch.equal(x.view(torch.int32), y.view(torch.int32))
