"""Host-side arithmetic of the 27B-shape decode pass (yskn_b200/stack.py): the layer pattern,
the code bytes of the stack against the reference's config-5 figure, the algorithmic bytes of
one token and the launch count (436 per token with the chain between projections inside the
operators, 660 with separate calls)."""
import types

from yskn_b200 import stack as S


def test_layer_pattern():
    kinds = S.layer_kinds(64)
    assert kinds.count("attn") == 16 and kinds.count("gdn") == 48
    assert [i for i, k in enumerate(kinds) if k == "attn"][:3] == [3, 7, 11]


def test_bytes():
    body = S.weight_bytes(64, S.VOCAB) - 2 * S.VOCAB * S.HIDDEN * 8 // 16
    # per layer: GDN 382,730,240 and attention 372,244,480 weights at 4 bits per weight
    assert body == (48 * 382_730_240 + 16 * 372_244_480) // 2
    tb = S.token_bytes(64, S.VOCAB, 4096)
    head = S.VOCAB * S.HIDDEN // 2
    assert tb == body + head + S.HIDDEN // 2 + 48 * (2 * 2 * 48 * 5120 + 8 * 48 * 128 * 128) + 16 * 1056 * 4097


def test_launches_per_token():
    fake = types.SimpleNamespace(kinds=S.layer_kinds(64), layers=64)
    assert S.Stack.launches_per_token(fake, fused=False) == 660
    # the chain inside the operators: no residual_prepare after the first layer's, no
    # separate quantiser for down (the MLP product is quantised in place), the GDN mixer
    # (gates, step, history) in one launch
    assert S.Stack.launches_per_token(fake) == 436
