"""The decode pass of the 27B-shape hybrid stack (yskn_b200/stack.py) on a short stack:
four layers (three Gated DeltaNet, one attention), a 4,096-row head and a 256-row KV cache.
Every call reports success, the greedy token stays inside the vocabulary, and the pass
captured as a CUDA graph produces the same tokens, hidden rows and recurrent states, bit
for bit, as the same pass run eagerly from the same starting state."""
import pytest

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
