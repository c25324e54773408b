"""The 27B-shape decode pass split over tensor-parallel ranks (one process per GPU).

The reference runs the whole pass on one GPU (src/engine35.cpp:768-842, :1268-1284); this
is the multi-GPU form of yskn_b200/stack.py, bit-identical to it token for token. Every
split follows the format's 512-blocks:

* Gated DeltaNet layers split by value head: out_proj's input columns (whole 512-groups,
  four value heads each) give a rank its value heads; the rank runs in_proj_qkv's query and
  key rows of the key heads they read (whole 512-row blocks, so a key head can run on two
  ranks) and the value rows of its heads, in_proj_z's rows of its heads, the dense gates,
  convolution, recurrent states and history of those channels (yskn_b200_gdn_*_heads).
* Attention layers split by query head: o_proj's input columns (512-groups, two query
  heads each) give a rank its query heads; it runs their q_proj rows (query and gate) and
  the KV heads they read (k_proj / v_proj rows in 512-blocks of two KV heads), keeping
  those heads' caches; with a fixed split count the attention's bits do not depend on how
  many heads a launch holds.
* The MLP splits gate/up by 512-row blocks and down by the same 512-column groups.
* o_proj, out_proj and down are row-parallel: one launch per rank with the exchange over
  NVLink inside the kernel (yskn_b200_linear_rowpar, _rowpar_q8 for down's quantised
  input), the whole projection on every rank; the next operator adds it to the residual
  stream in its own launch on every rank, so the stream is the same bits everywhere.
* The head splits over vocabulary rows; each rank's first eight are gathered (NCCL) and
  merged (yskn_b200_head_merge) into the same greedy token on every rank.

Weights are the stack's seeded tensors: every rank draws the whole tensor in the same order
as one GPU does and keeps its part, so the pass equals the one-GPU pass.
"""
import contextlib

import numpy as np
import torch
import torch.distributed as dist

import yskn_b200 as Y
from yskn_b200 import stack as S
from yskn_b200.tp import make_exchange, split_blocks

DK = 128               # Gated DeltaNet channels per head
QK = 16 * DK           # query (and key) channels of in_proj_qkv
GDN_RATIO = 48 // 16   # value heads per key head
KV_GROUP = S.N_QH // S.N_KVH


class TPPlan:
    """The heads, rows and columns rank `rank` of `world` runs (host arithmetic only)."""

    def __init__(self, rank, world, vocab=S.VOCAB):
        self.rank, self.world = rank, world
        # Gated DeltaNet: out_proj's input groups set the value heads.
        c0, c1 = split_blocks(S.ZDIM, world)[rank]
        self.gdn_cols = (c0, c1)
        self.v0, self.n_v = c0 // DK, (c1 - c0) // DK
        k_lo, k_hi = self.v0 // GDN_RATIO, (self.v0 + self.n_v - 1) // GDN_RATIO + 1  # key heads read
        b0, b1 = k_lo * DK // 512, -(-k_hi * DK // 512)
        self.qk0, self.qk_ch = b0 * 512 // DK, (b1 - b0) * 512
        self.qkv_ranges = [(b0 * 512, b1 * 512), (QK + b0 * 512, QK + b1 * 512), (2 * QK + c0, 2 * QK + c1)]
        # Attention: o_proj's input groups set the query heads; their KV heads follow.
        a0, a1 = split_blocks(S.N_QH * S.HEAD, world)[rank]
        self.attn_cols = (a0, a1)
        self.h0, self.n_q = a0 // S.HEAD, (a1 - a0) // S.HEAD
        self.kv0 = self.h0 // KV_GROUP
        self.n_kv = (self.h0 + self.n_q - 1) // KV_GROUP + 1 - self.kv0
        kb0, kb1 = self.kv0 // 2, -(-(self.kv0 + self.n_kv) // 2)  # k/v blocks: two KV heads each
        self.kv_rows = (kb0 * 512, kb1 * 512)
        self.kv_skip = self.kv0 - 2 * kb0  # KV heads of the local k/v output before the first used
        self.q_rows = (self.h0 * 2 * S.HEAD, (self.h0 + self.n_q) * 2 * S.HEAD)
        # MLP and head.
        self.ffn = split_blocks(S.FFN, world)[rank]
        self.vocab_ranges = split_blocks(vocab, world)
        self.vocab = self.vocab_ranges[rank]

    def check(self):
        """The local head mappings the kernels assume: query head j of the rank reads local KV
        head j / (n_q / n_kv); value head v0 + i reads a key head among the rank's."""
        ratio = self.n_q // self.n_kv
        assert self.n_q % self.n_kv == 0
        for j in range(self.n_q):
            assert (self.h0 + j) // KV_GROUP - self.kv0 == j // ratio
        assert self.v0 // GDN_RATIO >= self.qk0
        assert (self.v0 + self.n_v - 1) // GDN_RATIO < self.qk0 + self.qk_ch // DK
        return self

    def shard(self, role, rows, cols):
        """Matrix shard argument of Y.Matrix for projection `role`."""
        if role == "qkv":
            return (self.qkv_ranges, 0, cols)
        if role == "z":
            return (*self.gdn_cols, 0, cols)
        if role == "out":
            return (0, rows, *self.gdn_cols)
        if role == "q":
            return (*self.q_rows, 0, cols)
        if role in ("k", "v"):
            return (*self.kv_rows, 0, cols)
        if role == "o":
            return (0, rows, *self.attn_cols)
        if role in ("gate", "up"):
            return (*self.ffn, 0, cols)
        if role == "down":
            return (0, rows, *self.ffn)
        if role == "head":
            return (*self.vocab, 0, cols)
        raise ValueError(role)

    def channels(self, a, axis=-1):
        """The rank's in_proj_qkv channels of a per-channel array (query, key, value runs)."""
        idx = np.concatenate([np.arange(r0, r1) for r0, r1 in self.qkv_ranges])
        return a.index_select(axis if axis >= 0 else a.dim() + axis, torch.as_tensor(idx, device=a.device))


class TPStack(S.Stack):
    """One rank's part of the stack (S.Stack's tensors, drawn whole and cut by TPPlan)."""

    def __init__(self, device, layers=64, vocab=S.VOCAB, ctx=4096, bits=8, seed=1, kinds=None, group=None):
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        self.plan = TPPlan(rank, world, vocab).check()
        self.group = group
        super().__init__(device, layers=layers, vocab=vocab, ctx=ctx, bits=bits, seed=seed, kinds=kinds)
        P = self.plan
        f32 = lambda *s: torch.zeros(s, dtype=torch.float32, device=device)  # noqa: E731
        i16 = lambda *s: torch.zeros(s, dtype=torch.int16, device=device)  # noqa: E731
        i8 = lambda *s: torch.zeros(s, dtype=torch.int8, device=device)  # noqa: E731
        for L in self.L:
            if L["kind"] == "gdn":
                v = slice(P.v0, P.v0 + P.n_v)
                L["wb"], L["wa"] = L["wb"][v].contiguous(), L["wa"][v].contiguous()
                L["a_log"], L["dt_bias"] = L["a_log"][v].contiguous(), L["dt_bias"][v].contiguous()
                L["state"] = L["state"][v].contiguous()
                L["conv"] = P.channels(L["conv"], axis=0).contiguous()
                L["history"] = P.channels(L["history"], axis=1).contiguous()
            else:
                kv = slice(P.kv0, P.kv0 + P.n_kv)
                L["cache"] = L["cache"][:, kv].contiguous()
                L["scales"] = L["scales"][:, kv].contiguous()
        torch.cuda.empty_cache()
        W = 2 * P.qk_ch + DK * P.n_v
        self.qkv_o, self.z_o = f32(1, W), f32(1, DK * P.n_v)
        self.gates, self.g_out = f32(1, 2 * P.n_v), f32(1, DK * P.n_v)
        kv_blocks = (P.kv_rows[1] - P.kv_rows[0]) // S.HEAD
        self.q_o = f32(1, P.n_q, 2 * S.HEAD)
        self.k_o, self.v_o = f32(1, kv_blocks, S.HEAD), f32(1, kv_blocks, S.HEAD)
        self.query, self.a_gate, self.a_out = (i16(1, P.n_q, S.HEAD) for _ in range(3))
        self.kv_rows = f32(2 * P.n_kv, S.HEAD)
        self.a_in = f32(1, P.n_q * S.HEAD)
        n_ffn = P.ffn[1] - P.ffn[0]
        self.g_o, self.u_o = f32(1, n_ffn), f32(1, n_ffn)
        self.act_m, self.alpha_m = i8(1, n_ffn), f32(1, n_ffn // 512)
        self.logits = f32(1, P.vocab[1] - P.vocab[0])
        t = lambda a: torch.as_tensor(np.ascontiguousarray(a), device=device)  # noqa: E731
        self.kv_groups = t(np.array([side * S.N_KVH + P.kv0 + h for side in range(2) for h in range(P.n_kv)], np.int32))
        self.kv_dest = t(np.array([h * (ctx + 1) + ctx for h in range(2 * P.n_kv)], np.int64))
        self.kv_book = self.kv_book[:P.n_kv].contiguous()
        # The one-GPU pass's split count (one wave of the device's SMs over the four KV heads),
        # fixed, so a launch over fewer heads adds up the same splits.
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        self.kv_splits = max(1, min(64, sms // S.N_KVH))
        self.kv_work = torch.empty(max(16, Y.kv4_attention_work_bytes(1, P.n_q, ctx + 1, self.kv_splits)),
                                   dtype=torch.uint8, device=device)
        first = [self.L[0]["qkv"], self.L[0]["z"]] if self.L[0]["kind"] == "gdn" else \
            [self.L[0]["q"], self.L[0]["k"], self.L[0]["v"]]
        self.work = torch.empty(Y.linear_work_bytes(first, 1), dtype=torch.uint8, device=device)
        # the head's exchange: this rank's first eight (logits, then ids as int32 bits)
        self.cand = torch.zeros((2, 1, 8), dtype=torch.int32, device=device)
        self.gathered = torch.zeros((world, 2, 1, 8), dtype=torch.int32, device=device)
        self.offsets = [r0 for r0, _ in P.vocab_ranges]
        self.exchange = make_exchange(S.HIDDEN, group=group)

    def _place(self, words, rows, cols, lut16, sc16, rotate, role):
        m = Y.Matrix(words, "warp", rows, rows, cols, self.bits, lut16, sc16, self._sign(0, cols),
                     self._sign(cols, rows) if rotate else None, shard=self.plan.shard(role, rows, cols))
        return m  # the whole tensor's words are dropped

    def close(self):
        """Unmaps the exchange; every rank calls it with no kernels in flight."""
        if self.exchange is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            self.exchange.close()
            self.exchange = None

    def decode(self, stream=None, fused=True):
        """One token on this rank: S.Stack.decode's fused chain with this rank's part of each
        step; every rank issues the same launches and collectives in order and ends with the
        same greedy token."""
        if not fused:
            raise ValueError("the tensor-parallel pass runs the fused chain only")
        return super().decode(stream)

    # The one-GPU pass (S.Stack.decode) with this rank's parts of each step.
    def _gdn(self, L, s):
        P = self.plan
        Y.gdn_mixer_heads(self.xg, self.inv, L["wb"], L["wa"], self.qkv_o, self.z_o, L["conv"], L["a_log"],
                          L["dt_bias"], L["norm_w"], S.EPS, L["state"], L["history"], self.g_out, P.v0, P.qk0,
                          P.qk_ch, stream=s)

    def _project(self, mat, x, s):
        """Row-parallel: this rank's input columns; the whole projection on every rank."""
        Y.linear_rowpar(self.exchange, mat, x, self.proj, stream=s)

    def _project_q8(self, mat, s):
        Y.linear_rowpar_q8(self.exchange, mat, self.act_m, self.alpha_m, self.proj, stream=s)

    def _select(self, s):
        """This rank's first eight of its vocabulary part, gathered from every rank and merged."""
        Y.head_select(self.logits, top_logits=self.cand[0].view(torch.float32), top_ids=self.cand[1], stream=s)
        with torch.cuda.stream(s) if s is not None else contextlib.nullcontext():
            dist.all_gather_into_tensor(self.gathered, self.cand, group=self.group)
        g = self.gathered
        Y.head_merge(g[:, 0].view(torch.float32), g[:, 1], self.offsets, token=self.token, stream=s)

    def _attention(self, L, s):
        P = self.plan
        k_use = self.k_o[:, P.kv_skip:P.kv_skip + P.n_kv]
        v_use = self.v_o[:, P.kv_skip:P.kv_skip + P.n_kv]
        Y.attention_prep(self.q_o, k_use, v_use, L["q_norm"], L["k_norm"], self.positions, S.EPS, self.query,
                         self.a_gate, self.kv_rows[:P.n_kv].view(1, P.n_kv, S.HEAD),
                         self.kv_rows[P.n_kv:].view(1, P.n_kv, S.HEAD), stream=s)
        cache, scales = L["cache"], L["scales"]
        Y.kv_encode(self.kv_rows, self.kv_groups, self.kv_tables, self.kv_gains, self.kv_mults, 4, True,
                    cache.view(-1, 32), scales.view(-1), dest=self.kv_dest, stream=s)
        Y.kv4_attention(self.query, cache[0], scales[0], cache[1], scales[1], self.kv_book, self.kv_book,
                        self.ctx + 1, self.kv_work, self.a_out, gate=self.a_gate, n_splits=self.kv_splits, stream=s)
        Y.widen_bf16(self.a_out.view(1, -1), self.a_in, stream=s)

    def launches_per_token(self, fused=True):
        """The one-GPU pass's launches plus the head merge (the gather is NCCL's)."""
        return super().launches_per_token(fused=True) + 1
