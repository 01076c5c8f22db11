"""Several positions of one sequence in one chalot_forward_batch, and greedy
speculative decoding built on it (src/model/speculative.rs:100-249: a draft
proposes k tokens, the model verifies them). The verified output must be the
model's own greedy tokens, whatever the draft proposes."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_rows_of_one_sequence_match_one_by_one(chalot, tiny_model):
    """Positions 0..n-1 of one sequence as rows of one call give the argmax and
    logits of n single-row calls, bit for bit."""
    toks = np.random.default_rng(5).integers(0, 4096, 12).tolist()
    a = chalot.Engine.load(tiny_model)
    b = chalot.Engine.load(tiny_model)
    try:
        a.reserve_batch(16)
        b.reserve_batch(16)
        one = [a.forward_batch([0], [t], [p])[0] for p, t in enumerate(toks)]
        la = a.batch_logits(0)
        many = b.forward_batch([0] * len(toks), toks, range(len(toks)))
        lb = b.batch_logits(len(toks) - 1)
        assert many == one
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    finally:
        a.close()
        b.close()


def test_repeated_slot_position_rejected(chalot, tiny_model):
    from chalot_c1_b200._capi import ChalotError
    e = chalot.Engine.load(tiny_model)
    try:
        e.reserve_batch(4)
        with pytest.raises(ChalotError, match="pair appears twice"):
            e.forward_batch([0, 0], [1, 2], [3, 3])
    finally:
        e.close()


@pytest.mark.parametrize("k", [1, 4])
def test_speculative_same_model_accepts_all(chalot, tiny_model, k):
    prompt = np.random.default_rng(6).integers(0, 4096, 10).tolist()
    ref = chalot.Engine.load(tiny_model)
    main = chalot.Engine.load(tiny_model)
    draft = chalot.Engine.load(tiny_model)
    try:
        want = ref.generate(prompt, 24)
        got, acc, prop = main.generate_speculative(prompt, 24, draft, k=k)
        assert got == want
        assert acc == prop  # the draft is the model itself
    finally:
        for e in (ref, main, draft):
            e.close()


def test_speculative_other_draft_keeps_greedy_tokens(chalot, tiny_model, tmp_path):
    """A draft with other weights (same vocabulary) is mostly rejected; the
    output is still the model's greedy sequence."""
    dpath = chalot.write_shape(str(tmp_path / "draft.myai"), "tiny", n_layers=2, seed=7)
    prompt = np.random.default_rng(7).integers(0, 4096, 9).tolist()
    ref = chalot.Engine.load(tiny_model)
    main = chalot.Engine.load(tiny_model)
    draft = chalot.Engine.load(dpath)
    try:
        want = ref.generate(prompt, 30)
        got, acc, prop = main.generate_speculative(prompt, 30, draft, k=3)
        assert got == want
        assert acc < prop
    finally:
        for e in (ref, main, draft):
            e.close()
