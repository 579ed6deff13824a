"""Step-graph cache under pressure on a B200: more launch plans than the four cached ones (six
batch sizes in rotation), so plans are evicted and captured again, with profiling (which
runs the stream form) switched on and off in between. Every step must match a context that
uses stream launches only. All batches are at most 8 slots, run on the fixed-order mma.sync
path (exact_max_batch=8), so the two contexts' logits are bit-identical."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_step_graph_eviction_and_profiling(pkg, tiny_gguf, cuda):
    kw = dict(max_batch=8, max_ctx=64, kv_bf16=True, exact_max_batch=8)
    ref = pkg.DecodeContext(tiny_gguf, **kw)
    gra = pkg.DecodeContext(tiny_gguf, **kw)
    gra.step_graph(True)
    rng = np.random.default_rng(21)
    sizes = [1, 2, 3, 4, 5, 6]
    for step in range(30):
        B = sizes[step % len(sizes)]
        if step == 12:
            gra.profile(True)
        if step == 18:
            gra.profile(False)
        toks = rng.integers(0, 32000, size=B)
        lr, nr = ref.decode_step(toks)
        lg, ng = gra.decode_step(toks)
        assert np.array_equal(lg, lr), step
        assert np.array_equal(ng, nr), step
    # six plans through four cache entries: every rotation re-captures, except while profiling
    caps = gra.step_graph_captures()
    assert caps >= 24 - 6, caps
    assert [gra.get_pos(b) for b in range(8)] == [ref.get_pos(b) for b in range(8)]
    ref.close()
    gra.close()
