"""GPU tests of the prefix cache (the reference's LZPrefixCache on token
ids, src/generate.c:3209-3390) and the resumed generation it feeds: a hit
restores the checkpointed recurrent state and forwards only the new tokens,
and the state it leaves gives the same verify logits, bit for bit, as
forwarding the whole prefix from a reset state; the counters and the
refusals (an unsplittable render, a mismatching prefix, a state reset
since the save) follow the reference."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_prefix_cache_turns(mini_dir):
    import lz98
    m = lz98.Model(mini_dir)
    s = lz98.State(m, 512, 4)
    pc = lz98.PrefixCache(m)
    rng = np.random.default_rng(31)
    P = rng.integers(0, m.vocab, 30).astype(np.int32)
    T1 = rng.integers(0, m.vocab, 5).astype(np.int32)
    # turn 1: nothing cached, the whole prefix is forwarded and saved
    sp, ru = pc.prepare(s, np.concatenate([P, T1]), P, T1)
    assert (sp, ru) == (30, 0)
    toks1, _ = s.generate_resume(sp, T1, 12, 2)
    fresh = lz98.State(m, 512, 4)
    full1, _ = fresh.generate(np.concatenate([P, T1]), 12, 2)
    assert np.array_equal(toks1, full1)     # greedy: the emitted stream does not depend on the drafts
    # turn 2: the conversation grew; its prefix extends turn 1's
    P2 = np.concatenate([P, T1, toks1[:6]]).astype(np.int32)
    T2 = rng.integers(0, m.vocab, 4).astype(np.int32)
    assert pc.match(P2) == 30
    sp, ru = pc.prepare(s, np.concatenate([P2, T2]), P2, T2)
    assert (sp, ru) == (len(P2), 30)
    hv, lv = s.verify(T2, sp)
    fresh.reset()
    fresh.batch_capture(P2, 0)
    hv0, lv0 = fresh.verify(T2, len(P2))
    assert np.array_equal(bits(lv), bits(lv0)) and np.array_equal(bits(hv), bits(hv0))
    st = pc.stats()
    assert st == {"calls": 2, "hits": 1, "tokens_saved": 30, "mismatch": 0, "unsplittable": 0}
    # a render that does not split token-exactly takes the full path and drops the cache
    sp, ru = pc.prepare(s, np.concatenate([P2, T2]), P2, T2[::-1].copy())
    assert (sp, ru) == (0, 0) and pc.stats()["unsplittable"] == 1 and pc.match(P2) == 0
    # a mismatching conversation: counted, nothing reused
    sp, ru = pc.prepare(s, np.concatenate([P2, T2]), P2, T2)   # re-caches P2 (miss after the drop)
    Q = rng.integers(0, m.vocab, 20).astype(np.int32)
    sp, ru = pc.prepare(s, np.concatenate([Q, T2]), Q, T2)
    assert ru == 0 and sp == 20 and pc.stats()["mismatch"] == 1
    # a state reset since the save: the checkpoint is stale, nothing reused
    s.reset()
    sp, ru = pc.prepare(s, np.concatenate([Q, T2]), Q, T2)
    assert (sp, ru) == (20, 0)
    pc.close()
    fresh.close()
    s.close()
    m.close()
