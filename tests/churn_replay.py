"""Test helpers for the churn driver: a host-only pool with the
all-or-nothing batch reservation of s1kv_batch_begin, and the replay of a
driver's bookkeeping log on the oracle pool."""
import contextlib


class HostBatchPool:
    """A host-only s1kv.Pool whose batch() reserves every sequence's tokens
    or none: on S1KV_ENOBLOCKS the sequences touched so far are truncated
    back (or removed if the call created them) in reverse order, as
    s1kv_batch_begin does."""

    def __init__(self, pool):
        self.p = pool

    def __getattr__(self, name):
        return getattr(self.p, name)

    def batch(self, seqs, n_append, q_lens):
        import s1kv
        done = []
        for s, n in zip(seqs, n_append):
            done.append((s, self.p.length(s), self.p.exists(s)))
            st, _ = self.p.reserve(s, n)
            if st != 0:
                for s2, old, existed in reversed(done):
                    if existed:
                        self.p.truncate(s2, old)
                    elif self.p.exists(s2):
                        self.p.remove(s2)
                raise s1kv.S1KVError(st, "no blocks")
        return contextlib.nullcontext()


def replay(log, opool):
    """Applies a ChurnDriver log to an oracle.Pool (same operations, same
    rollback of failed batches)."""
    for op in log:
        kind = op[0]
        if kind == "remove":
            assert opool.remove(op[1]) == 0
        elif kind == "match":
            rc, _ = opool.prefix_match(op[1], op[2])
            assert rc == 0
        elif kind == "insert":
            opool.prefix_insert(op[1], op[2])
        elif kind in ("batch", "batch_fail"):
            done, failed = [], False
            for s, n in zip(op[1], op[2]):
                done.append((s, opool.length(s), opool.has(s)))
                rc, _, _ = opool.reserve(s, n)
                if rc != 0:
                    failed = True
                    for s2, old, existed in reversed(done):
                        if existed:
                            opool.truncate(s2, old)
                        elif opool.has(s2):
                            opool.remove(s2)
                    break
            assert failed == (kind == "batch_fail"), op[:1]
        else:
            raise ValueError(kind)
