"""The DDTreeBranchCache mirror (kgcuda.DDTreeBranchCache, after
src/speculative/types.rs:218-290) driven against a stand-in backend whose
paged calls go to the oracle's PagedKVCache: the branch budget, the trunk,
discard and reset behave as the reference's (no GPU needed; the device side of
the same calls is tests/test_gpu_paged.py)."""
import numpy as np


class OraclePagedBackend:
    def __init__(self, orc, cfg, w):
        self.orc, self.cfg, self.w = orc, cfg, w
        self.cache = None

    def paged_init(self, n):
        self.cache = self.orc.PagedKVCache(self.cfg, n)

    def paged_fork(self, seq, pos):
        return self.cache.fork(seq, pos)

    def paged_rollback(self, seq, pos):
        self.cache.rollback(seq, pos)

    def paged_reset(self):
        self.cache.reset()

    def forward(self, token, pos, seq=0):
        return self.orc.forward_paged(self.cfg, self.w, self.cache, seq, token, pos)


def test_branch_budget_fork_discard_reset(kg, orc):
    cfg = orc.config()
    be = OraclePagedBackend(orc, cfg, orc.weights(cfg, 42))
    tree = kg.DDTreeBranchCache(be, max_branches=3)
    for pos, tok in enumerate([26, 3, 9, 14]):
        logits = tree.forward_branch(0, tok, pos)
        assert logits.shape == (cfg.vocab_size,) and np.all(np.isfinite(logits))
    a = tree.fork_branch(0, 4)
    b = tree.fork_branch(0, 2)
    assert (a, b) == (3, 4)                       # indices after the 3 initial sequences
    assert tree.fork_branch(0, 4) == 0            # budget exhausted: the source comes back
    tree.forward_branch(a, 7, 4)
    tree.rollback_branch(a, 0)
    assert be.cache.layer_page_tables[0][a] == []
    tree.discard_branch(b)
    assert tree.branch_count == 2
    assert tree.fork_branch(0, 4) == 5            # a slot of the budget is free again
    tree.discard_branch(0)                        # the trunk does not give back a slot
    assert tree.branch_count == 3
    tree.reset()
    assert tree.branch_count == 1 and all(len(t) == 0 for t in be.cache.layer_page_tables[0])
