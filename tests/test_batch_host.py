"""Host-side scheduling of the batched forward, with a fake device: the
number of chalot_forward_batch calls per rank (expert-parallel ranks must make
the same number), the greedy bookkeeping of generate_batch, and the
draft/verify bookkeeping of generate_speculative. The fake engine keeps each
slot's tokens by position, as the KV cache does (a later write to a position
replaces it), and its "argmax" after position p is a fixed function of the
slot's tokens 0..p, so stale entries would change the answer."""
import zlib

import pytest

from chalot_c1_b200.engine import Engine


def _next(tokens, vocab, salt=0):
    return zlib.crc32(bytes(str((salt,) + tuple(tokens)), "ascii")) % vocab


class FakeEngine(Engine):
    def __init__(self, vocab=50, salt=0, wrong_every=0, max_seq=4096):
        self._h = None
        self._ep = None
        self._cap = 0
        self.config = {"vocab_size": vocab, "max_seq_len": max_seq}
        self.salt, self.wrong_every, self.calls, self.kv = salt, wrong_every, 0, {}

    def close(self):
        pass

    def reserve_batch(self, max_seqs):
        self._cap = max(self._cap, max_seqs)

    def forward_batch(self, slots, tokens, positions):
        slots, tokens, positions = list(slots), list(tokens), list(positions)
        assert len(slots) <= self._cap
        self.calls += 1
        for s, t, p in zip(slots, tokens, positions):  # every row's K/V before any row attends
            self.kv.setdefault(s, {})[p] = t
        out = []
        for s, p in zip(slots, positions):
            hist = [self.kv[s][q] for q in range(p + 1)]
            v = _next(hist, self.config["vocab_size"], self.salt)
            if self.wrong_every and (p % self.wrong_every == 0):
                v = (v + 1) % self.config["vocab_size"]  # a draft that is sometimes wrong
            out.append(v)
        return out


def _greedy(prompt, n, vocab=50):
    seq, out = list(prompt) or [0], []
    for _ in range(n):
        t = _next(seq, vocab)
        out.append(t)
        seq.append(t)
    return out


def test_generate_batch_greedy_and_call_count():
    prompts = [[1, 2, 3], [4], [5, 6, 7, 8, 9]]
    e = FakeEngine()
    got = e.generate_batch(prompts, 6)
    assert got == [_greedy(p, 6) for p in prompts]
    assert e.calls == Engine.batch_steps(prompts, 6)


def test_generate_batch_pads_calls_for_a_group():
    prompts = [[1, 2], [3]]
    e = FakeEngine()
    e._ep = (0, 2)  # as attached: empty calls continue to the group's count
    steps = Engine.batch_steps(prompts, 4) + 5
    got = e.generate_batch(prompts, 4, steps=steps)
    assert got == [_greedy(p, 4) for p in prompts]
    assert e.calls == steps
    idle = FakeEngine()
    idle._ep = (1, 2)
    assert idle.generate_batch([], 4, reserve=2, steps=steps) == []
    assert idle.calls == steps
    with pytest.raises(ValueError):
        FakeEngine().generate_batch(prompts, 4, steps=1)


@pytest.mark.parametrize("k", [1, 3, 5])
@pytest.mark.parametrize("wrong_every", [0, 2, 3])
def test_speculative_bookkeeping(k, wrong_every):
    prompt = [7, 8, 9, 10]
    main = FakeEngine()
    draft = FakeEngine(wrong_every=wrong_every)  # same function, wrong at some positions
    got, acc, prop = main.generate_speculative(prompt, 17, draft, k=k)
    assert got == _greedy(prompt, 17)
    if wrong_every == 0:
        assert acc == prop
    else:
        assert acc < prop


def test_speculative_unrelated_draft():
    prompt = [3, 1, 4, 1, 5]
    main, draft = FakeEngine(), FakeEngine(salt=99)
    got, acc, prop = main.generate_speculative(prompt, 12, draft, k=4)
    assert got == _greedy(prompt, 12)
