"""Between-block rank liveness for multi-rank stacks (host side).

The reference stops a denoise step between blocks through its progress
callback (Ltx25Dit's `in.progress`, src/ltx25-dit.cc:1718-1720) and runs on
one device.  Over several ranks a stop has to be a shared decision: a rank
that enqueues block i's all-reduce while a peer has stopped (exited, crashed,
never joined, or asked to abort) waits on the GPU for a contribution that
never comes.  RankWatch is that progress callback made collective, through
any torch.distributed Store (TCPStore, FileStore, HashStore):

* before block i each rank commits to it (an atomic counter per rank), unless
  an abort was already requested;
* it then waits, at most `timeout_s`, until every peer has committed to the
  same check;
* the first rank to see every commitment writes "go" for that check, the
  first to give up (bound reached, abort requested) writes "stop", both by
  compare_set, so exactly one decision exists per check and every live rank
  follows it: all of them enqueue block i, or none does.

A rank that dies after committing and before its own collective is past what
a host check can see; the process group's (or NCCL's) timeout bounds that
case.  Use: `watch = RankWatch(store, rank, world)`, then
`stack.forward(video, audio, progress=watch)` on every rank.
"""
import time

__all__ = ["RankWatch"]


class RankWatch:
    """progress(block, blocks) -> bool for `Stack.forward`, agreed over ranks.

    `failed` is None while every check went ahead, else (rank, reason): the
    peer that lagged past the bound or asked to abort (-1 when unknown) and
    why.  Once a check has stopped, every later call returns False.
    """

    def __init__(self, store, rank, world, timeout_s=30.0, prefix="ltx25/watch",
                 poll_s=0.0005):
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside a world of {world}")
        if timeout_s <= 0:
            raise ValueError("timeout_s must be positive")
        self.store = store
        self.rank = rank
        self.world = world
        self.timeout_s = float(timeout_s)
        self.prefix = prefix
        self.poll_s = float(poll_s)
        self.seq = 0
        self.failed = None

    def _key(self, *parts):
        return "/".join((self.prefix,) + tuple(str(p) for p in parts))

    def abort(self, reason=""):
        """Ask every rank to stop before its next block (this one included)."""
        self.store.compare_set(self._key("abort"), "", f"{self.rank}:{reason}")

    def aborted(self):
        """(rank, reason) of the first abort request, or None."""
        key = self._key("abort")
        if not self.store.check([key]):
            return None
        who, _, why = self.store.get(key).decode().partition(":")
        return int(who), why

    def _decide(self, seq, value):
        # the first writer wins; everybody reads back the one decision
        return self.store.compare_set(self._key("decision", seq), "", value).decode()

    def _follow(self, seq, decision):
        if decision == "go":
            if self.rank == 0 and seq > 2:
                # every rank read decision seq - 2 before committing to seq - 1
                try:
                    self.store.delete_key(self._key("decision", seq - 2))
                except (RuntimeError, NotImplementedError):
                    pass
            return True
        _, who, why = decision.split(":", 2)
        self.failed = (int(who), why)
        return False

    def _stop(self, seq):
        a = self.aborted()
        if a is not None:
            return self._decide(seq, f"stop:{a[0]}:abort requested: {a[1]}")
        lag = [p for p in self._lagging(seq)]
        who = lag[0] if lag else -1
        return self._decide(seq, f"stop:{who}:no commitment within {self.timeout_s:g} s "
                                 f"(check {seq})")

    def _lagging(self, seq):
        return [p for p in range(self.world)
                if p != self.rank and self.store.add(self._key("pos", p), 0) < seq]

    def __call__(self, block=None, blocks=None):
        if self.failed is not None:
            return False
        self.seq += 1
        seq = self.seq
        if self.aborted() is not None:
            # not committed: no "go" can exist for this check
            return self._follow(seq, self._stop(seq))
        self.store.add(self._key("pos", self.rank), 1)
        dkey = self._key("decision", seq)
        deadline = time.monotonic() + self.timeout_s
        while True:
            if self.store.check([dkey]):
                return self._follow(seq, self.store.get(dkey).decode())
            if not self._lagging(seq):
                return self._follow(seq, self._decide(seq, "go"))
            if self.aborted() is not None or time.monotonic() > deadline:
                return self._follow(seq, self._stop(seq))
            time.sleep(self.poll_s)
