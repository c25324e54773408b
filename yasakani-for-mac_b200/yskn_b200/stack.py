"""The 27B-shape decode pass at batch 1, built from the library's calls.

The hybrid stack of the reference's headline model shape: `layers` layers, every fourth a
full-attention layer (24 query heads of 256 with gates, 4 KV heads, a 4-bit quantised
cache) and the others Gated DeltaNet layers (16 q/k and 48 value heads of 128, recurrent
state), each followed by the gated MLP; hidden 5120, MLP 17408, coded embedding and head
over `vocab` rows; every compressed matrix at one trellis width (bits=8: 4 bits per
weight). One token runs as the reference's decode pass does (src/engine35.cpp:1268-1284,
layer order src/engine35.cpp:773-799): embedding row -> per layer (residual + norm ->
mixer -> residual + norm -> MLP) -> final norm -> head logits -> greedy token, the token
fed back on the device, so the pass is one CUDA graph per token.

Weights are seeded random code words generated on the device (every bit string is a
valid code) with synthetic value tables and row scales; norms, gates and convolution
weights are seeded bf16; the KV caches hold `ctx` synthetic rows and each token encodes
its own K/V row at position `ctx`. No model file is shipped with the reference.
"""
import numpy as np

import yskn_b200 as Y
from yskn_b200 import synthetic

HIDDEN, FFN, VOCAB = 5120, 17408, 151936
N_QH, N_KVH, HEAD = 24, 4, 256
QKV, ZDIM = 10240, 6144
EPS = 1e-6
SIGN_RULE = "mulberry32_7919_13"


def layer_kinds(layers):
    """'attn' for every fourth layer (3, 7, ...), else 'gdn' (src/engine35.cpp:255-263)."""
    return ["attn" if i % 4 == 3 else "gdn" for i in range(layers)]


def weight_bytes(layers, vocab, bits=8):
    """Code bytes of every compressed matrix of the stack (embedding and head included)."""
    per = {"gdn": [(QKV, HIDDEN), (ZDIM, HIDDEN), (HIDDEN, ZDIM)],
           "attn": [(N_QH * 2 * HEAD, HIDDEN), (N_KVH * HEAD, HIDDEN), (N_KVH * HEAD, HIDDEN), (HIDDEN, N_QH * HEAD)]}
    mlp = [(FFN, HIDDEN), (FFN, HIDDEN), (HIDDEN, FFN)]
    total = 2 * vocab * HIDDEN * bits // 16
    for k in layer_kinds(layers):
        total += sum(r * c * bits // 16 for r, c in per[k] + mlp)
    return total


def token_bytes(layers, vocab, ctx, bits=8):
    """Algorithmic bytes one token must move: every compressed matrix's codes except the
    embedding table (one row of it), the dense bf16 gate weights, each GDN state read and
    written, each attention layer's K/V cache rows (1,056 bytes per row: 4 heads x K, V x
    (128 + 4)), one new row encoded per attention layer."""
    kinds = layer_kinds(layers)
    gdn, attn = kinds.count("gdn"), kinds.count("attn")
    codes = weight_bytes(layers, vocab, bits) - vocab * HIDDEN * bits // 16 + HIDDEN * bits // 16
    return codes + gdn * (2 * 2 * 48 * HIDDEN + 2 * 4 * 48 * 128 * 128) + attn * 1056 * (ctx + 1)


class Stack:
    """Seeded weights, caches, states and buffers of the stack on one device."""

    def __init__(self, device, layers=64, vocab=VOCAB, ctx=4096, bits=8, seed=1, kinds=None):
        """kinds: an explicit list of layer kinds ('gdn' / 'attn'), else layer_kinds(layers)."""
        import torch
        self.torch, self.dev = torch, device
        self.layers, self.vocab, self.ctx, self.bits = layers, vocab, ctx, bits
        self.gen = torch.Generator(device=device)
        self.gen.manual_seed(seed)
        self.rng = np.random.default_rng(seed)
        self._signs = {}
        self._keep = []
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
        bfb = lambda a: t(self._bf16(a).view(np.int16))  # noqa: E731
        self.kinds = list(kinds) if kinds is not None else layer_kinds(layers)
        self.layers = layers = len(self.kinds)
        self.L = []
        for i, kind in enumerate(self.kinds):
            L = {"kind": kind, "in_norm": bfb(self._normal(HIDDEN) * 0.1), "post_norm": bfb(self._normal(HIDDEN) * 0.1),
                 "gate": self._matrix(FFN, HIDDEN, role="gate"), "up": self._matrix(FFN, HIDDEN, role="up"),
                 "down": self._matrix(HIDDEN, FFN, role="down")}
            if kind == "gdn":
                L.update(qkv=self._matrix(QKV, HIDDEN, role="qkv"), z=self._matrix(ZDIM, HIDDEN, role="z"),
                         out=self._matrix(HIDDEN, ZDIM, role="out"),
                         wb=bfb(self._normal(48 * HIDDEN).reshape(48, HIDDEN) * 0.02),
                         wa=bfb(self._normal(48 * HIDDEN).reshape(48, HIDDEN) * 0.02),
                         conv=bfb(self._normal(QKV * 4).reshape(QKV, 4) * 0.5),
                         a_log=bfb(self._normal(48) * 0.5), dt_bias=bfb(self._normal(48) * 0.5),
                         norm_w=bfb(1.0 + self._normal(128) * 0.1),
                         state=torch.zeros((48, 128, 128), dtype=torch.float32, device=device),
                         history=torch.zeros((3, QKV), dtype=torch.int16, device=device))
            else:
                cap = ctx + 1
                cache = torch.randint(-2 ** 31, 2 ** 31, (2, N_KVH, cap, 32), dtype=torch.int32, device=device,
                                      generator=self.gen)
                scales = 0.02 + 0.18 * torch.rand((2, N_KVH, cap), device=device, generator=self.gen)
                L.update(q=self._matrix(N_QH * 2 * HEAD, HIDDEN, role="q"), k=self._matrix(N_KVH * HEAD, HIDDEN, role="k"),
                         v=self._matrix(N_KVH * HEAD, HIDDEN, role="v"), o=self._matrix(HIDDEN, N_QH * HEAD, role="o"),
                         q_norm=bfb(self._normal(HEAD) * 0.1), k_norm=bfb(self._normal(HEAD) * 0.1),
                         cache=cache, scales=scales)
            self.L.append(L)
        self.final_norm = bfb(self._normal(HIDDEN) * 0.1)
        self.head = self._matrix(vocab, HIDDEN, rotate=False, role="head")
        emb_codes = torch.randint(-2 ** 31, 2 ** 31, (vocab * (HIDDEN // 256) * 4 * bits,), dtype=torch.int32,
                                  device=device, generator=self.gen)
        lut16, sc16 = synthetic.model_tables(vocab, int(self.rng.integers(1 << 30)))
        self._keep.append(emb_codes)
        self.embedding_source = (emb_codes, lut16, sc16)
        self.embedding = Y.Embedding([(emb_codes, bits, lut16, sc16)], vocab, HIDDEN, self._sign(0, HIDDEN))
        # the synthetic KV profile (the codebook of synthetic.kv_codebook_bf16): one table per
        # (side, head) group, multipliers 0.9 / 1.0 / 1.1
        codes = ((np.arange(256) * 73 + 19) % 2049 - 1024).astype(np.int16)
        self.kv_tables = t(np.tile(codes, (2 * N_KVH, 1)))
        self.kv_gains = t(np.full(2 * N_KVH, 257.0 / 256.0, np.float32))
        self.kv_mults = t(np.array([0.9, 1.0, 1.1], np.float32))
        self.kv_groups = t(np.arange(2 * N_KVH, dtype=np.int32))
        self.kv_dest = t(np.array([h * (ctx + 1) + ctx for h in range(2 * N_KVH)], np.int64))
        self.kv_book = t(np.tile(synthetic.kv_codebook_bf16(), (N_KVH, 1)).view(np.int16))
        self.positions = t(np.array([ctx], np.int32))
        # activations
        f32 = lambda *s: torch.zeros(s, dtype=torch.float32, device=device)  # noqa: E731
        i16 = lambda *s: torch.zeros(s, dtype=torch.int16, device=device)  # noqa: E731
        self.token = torch.zeros(1, dtype=torch.int32, device=device)
        self.h, self.xg = i16(1, HIDDEN), i16(1, HIDDEN)
        self.h_alt = i16(1, HIDDEN)  # the residual stream's second buffer (linear_from_residual)
        self.x, self.inv, self.proj = f32(1, HIDDEN), f32(1), f32(1, HIDDEN)
        self.qkv_o, self.z_o, self.gates, self.g_out = f32(1, QKV), f32(1, ZDIM), f32(1, 96), f32(1, ZDIM)
        self.q_o, self.k_o, self.v_o = f32(1, N_QH, 2 * HEAD), f32(1, N_KVH, HEAD), f32(1, N_KVH, HEAD)
        self.query, self.a_gate, self.a_out = i16(1, N_QH, HEAD), i16(1, N_QH, HEAD), i16(1, N_QH, HEAD)
        self.kv_rows = f32(2 * N_KVH, HEAD)
        self.a_in = f32(1, N_QH * HEAD)
        self.g_o, self.u_o, self.m_o = f32(1, FFN), f32(1, FFN), f32(1, FFN)
        # the MLP product quantised for down (yskn_b200_gated_product_q8): int8 rows, group scales
        i8 = lambda *s: torch.zeros(s, dtype=torch.int8, device=device)  # noqa: E731
        self.act_m, self.alpha_m = i8(1, FFN), f32(1, FFN // 512)
        self.logits = f32(1, vocab)
        first = {k: next(L for L in self.L if L["kind"] == k) for k in set(self.kinds)}
        sets = [[self.head], [first[self.kinds[0]]["gate"], first[self.kinds[0]]["up"]], [self.L[0]["down"]]]
        if "gdn" in first:
            sets += [[first["gdn"]["qkv"], first["gdn"]["z"]], [first["gdn"]["out"]]]
        if "attn" in first:
            sets += [[first["attn"]["q"], first["attn"]["k"], first["attn"]["v"]], [first["attn"]["o"]]]
        self.work = torch.empty(max(Y.linear_work_bytes(s, 1) for s in sets), dtype=torch.uint8, device=device)
        self.kv_work = torch.empty(max(16, Y.kv4_attention_work_bytes(1, N_QH, ctx + 1, -1)), dtype=torch.uint8,
                                   device=device)

    def _normal(self, n):
        return self.rng.standard_normal(n).astype(np.float32)

    @staticmethod
    def _bf16(a):
        u = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

    def _sign(self, offset, n):
        if (offset, n) not in self._signs:
            self._signs[(offset, n)] = Y.signs(SIGN_RULE, 7, offset, n)
        return self._signs[(offset, n)]

    def _matrix(self, rows, cols, rotate=True, role=None):
        torch = self.torch
        words = torch.randint(-2 ** 31, 2 ** 31, (rows * (cols // 256) * 4 * self.bits,), dtype=torch.int32,
                              device=self.dev, generator=self.gen)
        lut16, sc16 = synthetic.model_tables(rows, int(self.rng.integers(1 << 30)))
        return self._place(words, rows, cols, lut16, sc16, rotate, role)

    def _place(self, words, rows, cols, lut16, sc16, rotate, role):
        """The matrix this device runs of a seeded tensor (here the whole tensor; the
        tensor-parallel stack keeps its rank's rows or columns). role names the projection."""
        self._keep.append(words)
        m = Y.Matrix(words, "warp", rows, rows, cols, self.bits, lut16, sc16, self._sign(0, cols),
                     self._sign(cols, rows) if rotate else None)
        m.source = (words, lut16, sc16, rotate)  # what a checker needs to rebuild the matrix
        return m

    def decode(self, stream=None, fused=True):
        """One token: reads self.token, writes the next greedy token into it. fused: the
        chain between projections inside the operators (each operator that follows a
        residual add forms its input in its own launch: residual, normalisation and quantiser,
        yskn_b200_linear_from_residual; the MLP product quantised for down; the GDN mixer in
        one launch), else the separate residual_prepare / gated_product / gates calls; both
        give the same bits. The
        residual stream alternates between two buffers and ends each token in self.h."""
        if not fused:
            return self._decode_separate(stream)
        s = stream
        hs = [self.h, self.h_alt]
        cur = 0

        def from_residual(mats, norm, outs, gate=None, inv=None):
            nonlocal cur
            Y.linear_from_residual(mats, self.proj, hs[cur], hs[1 - cur], norm, EPS, outs, gate_out=gate,
                                   inv_rms_out=inv, stream=s)
            cur = 1 - cur

        self.embedding.lookup(self.token, self.h, stream=s)
        Y.residual_prepare(self.h, None, self.L[0]["in_norm"], EPS, self.x, self.inv, gate=self.xg, stream=s)
        for i, L in enumerate(self.L):
            if L["kind"] == "gdn":
                mats, outs = [L["qkv"], L["z"]], [self.qkv_o, self.z_o]
            else:
                mats, outs = [L["q"], L["k"], L["v"]], [self.q_o, self.k_o, self.v_o]
            if i == 0:
                Y.linear(mats, self.x, self.work, outs, inv_rms=self.inv, stream=s)
            else:
                from_residual(mats, L["in_norm"], outs, gate=self.xg, inv=self.inv)
            if L["kind"] == "gdn":
                self._gdn(L, s)
                self._project(L["out"], self.g_out, s)
            else:
                self._attention(L, s)
                self._project(L["o"], self.a_in, s)
            from_residual([L["gate"], L["up"]], L["post_norm"], [self.g_o, self.u_o])
            Y.gated_product_q8(self.g_o, self.u_o, L["down"].signs_in_ptr, self.act_m, self.alpha_m, stream=s)
            self._project_q8(L["down"], s)
        from_residual([self.head], self.final_norm, [self.logits])
        assert cur == 0  # an even number of residual adds per token: the stream ends in self.h
        self._select(s)

    def _gdn(self, L, s):
        """The Gated DeltaNet mixer between in_proj and out_proj: gates, step and history in
        one launch."""
        Y.gdn_mixer(self.xg, self.inv, L["wb"], L["wa"], self.qkv_o, self.z_o, L["conv"], L["a_log"], L["dt_bias"],
                    L["norm_w"], EPS, L["state"], L["history"], self.g_out, stream=s)

    def _project(self, mat, x, s):
        """A mixer's output projection into self.proj (f32 input)."""
        Y.linear([mat], x, self.work, [self.proj], stream=s)

    def _project_q8(self, mat, s):
        """The down projection into self.proj from the quantised MLP product."""
        Y.linear_q8([mat], self.act_m, self.alpha_m, [self.proj], stream=s)

    def _select(self, s):
        Y.head_select(self.logits, token=self.token, stream=s)

    def _attention(self, L, s):
        """The attention mixer between q/k/v and o: inputs, the new K/V rows into the cache,
        attention with the gate, the bf16 output widened to o_proj's f32 input."""
        Y.attention_prep(self.q_o, self.k_o, self.v_o, L["q_norm"], L["k_norm"], self.positions, EPS,
                         self.query, self.a_gate, self.kv_rows[:N_KVH].view(1, N_KVH, HEAD),
                         self.kv_rows[N_KVH:].view(1, N_KVH, HEAD), stream=s)
        cache, scales = L["cache"], L["scales"]
        Y.kv_encode(self.kv_rows, self.kv_groups, self.kv_tables, self.kv_gains, self.kv_mults, 4, True,
                    cache.view(-1, 32), scales.view(-1), dest=self.kv_dest, stream=s)
        Y.kv4_attention(self.query, cache[0], scales[0], cache[1], scales[1], self.kv_book, self.kv_book,
                        self.ctx + 1, self.kv_work, self.a_out, gate=self.a_gate, n_splits=-1, stream=s)
        Y.widen_bf16(self.a_out.view(1, -1), self.a_in, stream=s)

    def _decode_separate(self, stream=None):
        s = stream
        self.embedding.lookup(self.token, self.h, stream=s)
        proj = None
        for L in self.L:
            Y.residual_prepare(self.h, proj, L["in_norm"], EPS, self.x, self.inv, gate=self.xg, stream=s)
            if L["kind"] == "gdn":
                Y.linear([L["qkv"], L["z"]], self.x, self.work, [self.qkv_o, self.z_o], inv_rms=self.inv, stream=s)
                Y.gdn_gates(self.xg, self.inv, L["wb"], L["wa"], self.gates, stream=s)
                Y.gdn_step(self.qkv_o, self.z_o, self.gates, L["conv"], L["a_log"], L["dt_bias"], L["norm_w"], EPS,
                           L["state"], L["history"], self.g_out, stream=s)
                Y.linear([L["out"]], self.g_out, self.work, [self.proj], stream=s)
            else:
                Y.linear([L["q"], L["k"], L["v"]], self.x, self.work, [self.q_o, self.k_o, self.v_o],
                         inv_rms=self.inv, stream=s)
                Y.attention_prep(self.q_o, self.k_o, self.v_o, L["q_norm"], L["k_norm"], self.positions, EPS,
                                 self.query, self.a_gate, self.kv_rows[:N_KVH].view(1, N_KVH, HEAD),
                                 self.kv_rows[N_KVH:].view(1, N_KVH, HEAD), stream=s)
                cache, scales = L["cache"], L["scales"]
                Y.kv_encode(self.kv_rows, self.kv_groups, self.kv_tables, self.kv_gains, self.kv_mults, 4, True,
                            cache.view(-1, 32), scales.view(-1), dest=self.kv_dest, stream=s)
                Y.kv4_attention(self.query, cache[0], scales[0], cache[1], scales[1], self.kv_book, self.kv_book,
                                self.ctx + 1, self.kv_work, self.a_out, gate=self.a_gate, n_splits=-1, stream=s)
                Y.widen_bf16(self.a_out.view(1, -1), self.a_in, stream=s)
                Y.linear([L["o"]], self.a_in, self.work, [self.proj], stream=s)
            Y.residual_prepare(self.h, self.proj, L["post_norm"], EPS, self.x, self.inv, stream=s)
            Y.linear([L["gate"], L["up"]], self.x, self.work, [self.g_o, self.u_o], inv_rms=self.inv, stream=s)
            Y.gated_product(self.g_o, self.u_o, self.m_o, stream=s)
            Y.linear([L["down"]], self.m_o, self.work, [self.proj], stream=s)
            proj = self.proj
        Y.residual_prepare(self.h, proj, self.final_norm, EPS, self.x, self.inv, stream=s)
        Y.linear([self.head], self.x, self.work, [self.logits], inv_rms=self.inv, stream=s)
        Y.head_select(self.logits, token=self.token, stream=s)

    def launches_per_token(self, fused=True):
        """This library's kernel launches in decode(), one per call except the separate
        GDN step (step + history). Fused chain: embedding, the first layer's normalisation, head
        operator (with the last residual add), head select; per layer the mixer's input
        operator (with the residual add before it, after the first layer), the mixer's output
        operator, gate/up (with the residual add), the quantised product and down; GDN mixer
        in between: one launch (gates, step, history); attention:
        preparation, KV encode, attention, widening. Separate calls: embedding, final
        norm, head operator, head select; per layer the input norm and the MLP (post norm,
        gate/up operator, gated product, down operator); GDN mixer: operator, gates, step
        (2), out operator; attention mixer: operator, preparation, KV encode, attention,
        widening, o operator."""
        gdn, attn = self.kinds.count("gdn"), self.kinds.count("attn")
        if fused:
            return 4 + self.layers * 5 + gdn + attn * 4
        return 4 + self.layers * 5 + gdn * 5 + attn * 6
