"""Recurrent-state checkpoints (lz_ckpt_*, the reference's
src/forward_ckpt.c): save after a prefix, advance the state, restore, and
the same continuation reproduces the same logits bit for bit; the
refusals of the reference (empty, stale after a reset) keep their codes."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CKPT_EMPTY, CKPT_STALE = 21, 22


@pytest.fixture(scope="module", params=["tiny", "mini"])
def model(request):
    from conftest import model_dir
    import lz98
    m = lz98.Model(model_dir(request.param))
    yield m
    m.close()


def test_restore_reproduces_continuation(model):
    import lz98
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, model.vocab, 14).astype(np.int32)
    cont = rng.integers(0, model.vocab, 3).astype(np.int32)
    s = lz98.State(model, 256, 4)
    ck = lz98.Checkpoint(model)
    assert ck.restore(s) == (CKPT_EMPTY, -1)
    s.batch_capture(prompt, 0)
    assert ck.save(s, len(prompt)) == 0
    h1, l1 = s.verify(cont, len(prompt))          # advances the ring
    assert s.positions()[1] != 0
    rc, pos = ck.restore(s)
    assert rc == 0 and pos == len(prompt) and s.positions()[1] == 0
    h2, l2 = s.verify(cont, pos)
    assert np.array_equal(l1.view(np.uint32), l2.view(np.uint32))
    assert np.array_equal(h1.view(np.uint32), h2.view(np.uint32))
    s.reset()
    assert ck.restore(s)[0] == CKPT_STALE
    ck.close()
    s.close()


def test_restore_of_one_sequence_leaves_the_others(model):
    """Save and restore sequence 1 of a two-sequence state between greedy
    rounds: sequence 0's tokens match a control state that never restored,
    so the per-sequence slices of the ring and conv history are addressed
    right."""
    import lz98
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, model.vocab, 10 + 3 * b).astype(np.int32) for b in range(2)]
    toks = []
    for do_restore in (False, True):
        s = lz98.State(model, 256, 2, n_seq=2)
        for b in range(2):
            s.seq_prefill(b, prompts[b])
        ck = lz98.Checkpoint(model)
        assert ck.save(s, len(prompts[1]), seq=1) == 0
        seq0 = []
        for r in range(4):
            if do_restore and r == 2:
                assert ck.restore(s, seq=1) == (0, len(prompts[1]))
                assert s.positions(1)[1] == 0
            t, c = s.round_batch(2)
            seq0 += t[0, :c[0]].tolist()
        toks.append(seq0)
        ck.close()
        s.close()
    assert toks[0] == toks[1]
