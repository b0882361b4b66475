"""Incremental decoding (prefill into per-layer caches + one-token steps).

The property: the hidden state (and logits) of a token decoded at position n
equal those of a plain prefill over the n + 1 tokens at its last row. The
cached path runs the same kernels -- the q6 pack in the qkvg epilogue writing
into the cache, DSQG over the q6 cache with a query-row window, HISA selector
tiles restricted to the new rows (CTAs stay on the full launch's tile grid and
visit routed chunks in ascending order, so rows are unchanged), the packet's
EMA continued from its carried fp32 state -- so with DSQG's gather kernel on
both sides the results are bit-identical. By default a prefill whose length
is a multiple of 8 takes the resident-K/V DSQG kernel, which rounds
differently from the gather kernel a decode row takes; bf16 activations then
differ by rounding steps that grow over ten blocks, and final hidden states
(RMS ~1) and logits must agree within 0.15 max-abs and 0.02 mean-abs.
"""

import pytest
import torch


def _model():
    from dwarf_v2_b200.model import DwarfForCausalLM

    return DwarfForCausalLM(kv_cache="q6").eval().to(torch.bfloat16).cuda()


def _close(a, b, exact=False):
    if exact:
        assert torch.equal(a, b), (a.float() - b.float()).abs().max().item()
        return
    d = (a.float() - b.float()).abs()
    assert d.max().item() < 0.15 and d.mean().item() < 0.02, (d.max().item(), d.mean().item())


def test_decode_api_errors_without_gpu():
    from dwarf_v2_b200.model import DwarfForCausalLM

    with pytest.raises(NotImplementedError):
        DwarfForCausalLM().new_decode_state(1, 64, device="cpu")


@pytest.mark.gpu
@torch.no_grad()
@pytest.mark.parametrize("path", ["gather", ""])
def test_prefill_matches_forward_and_chunked_prefill(path, monkeypatch):
    monkeypatch.setenv("DWARF_DSQG_PATH", path)
    exact = path == "gather"
    model = _model()
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, model.config.vocab_size, (2, 300), generator=g).cuda()
    ref = model(ids, return_hidden=True)
    state = model.new_decode_state(2, 512)
    h = model.forward_cached(ids, state)
    assert state.length == 300
    _close(h, ref, exact)
    # two chunks: rows [0,137) then [137,300) (row_begin > 0 with many query rows)
    state2 = model.new_decode_state(2, 512)
    h1 = model.forward_cached(ids[:, :137], state2)
    h2 = model.forward_cached(ids[:, 137:], state2)
    _close(torch.cat([h1, h2], 1), ref, exact)
    state3 = model.new_decode_state(2, 512)
    h1 = model.forward_cached(ids[:, :160], state3)
    h2 = model.forward_cached(ids[:, 160:], state3)
    _close(torch.cat([h1, h2], 1), ref, exact)


@pytest.mark.gpu
@torch.no_grad()
@pytest.mark.parametrize("prompt,steps", [(1, 70), (150, 40), (2040, 8)])
def test_decode_steps_match_prefill_of_the_prefix(prompt, steps):
    model = _model()
    g = torch.Generator().manual_seed(prompt)
    ids = torch.randint(0, model.config.vocab_size, (2, prompt + steps), generator=g).cuda()
    logits, state = model.prefill(ids[:, :prompt], max_len=prompt + steps)
    _close(logits, model(ids[:, :prompt])[:, -1])
    checked = 0
    for n in range(prompt, prompt + steps):
        logits = model.decode_step(state, ids[:, n])
        assert state.length == n + 1 and int(state.pos) == n + 1
        # every step through 64 tokens, then a sample (each check is a prefill over n+1 tokens)
        if n < 64 or n % 7 == 0 or n == prompt + steps - 1:
            _close(logits, model(ids[:, :n + 1])[:, -1])
            checked += 1
    assert checked > 0
    with pytest.raises(ValueError):
        model.decode_step(state, ids[:, 0])  # the state is full


@pytest.mark.gpu
@torch.no_grad()
def test_decode_graph_replays_the_eager_step_bit_for_bit():
    """A captured step (positions read from the device) replayed across chunk and tile
    boundaries equals the eager step exactly, and both track the prefill."""
    model = _model()
    g = torch.Generator().manual_seed(5)
    prompt, steps = 120, 80
    ids = torch.randint(0, model.config.vocab_size, (3, prompt + steps), generator=g).cuda()
    _, eager = model.prefill(ids[:, :prompt], max_len=prompt + steps)
    _, graphed = model.prefill(ids[:, :prompt], max_len=prompt + steps)
    graph = model.capture_decode(graphed)
    assert graphed.length == prompt and int(graphed.pos) == prompt
    for n in range(prompt, prompt + steps):
        a = model.decode_step(eager, ids[:, n])
        b = graph.step(ids[:, n])
        assert torch.equal(a, b), n
    assert graphed.length == eager.length == prompt + steps
    _close(b, model(ids)[:, -1])
    with pytest.raises(ValueError):
        graph.step(ids[:, 0])
