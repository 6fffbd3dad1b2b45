"""P emulated ranks in one process, for running the product's collective
orchestration (vidax_b200.ulysses, vidax_b200.ulysses_qsplit) unchanged.

Each rank is a thread. `RankGroup` stands in for the `torch.distributed`
module those files import as `dist`: its all_to_all_single (equal or per-rank
split sizes), all_gather_into_tensor, get_rank and get_world_size exchange
the ranks' tensors through shared memory behind a barrier with a timeout (a
failing rank breaks the barrier instead of hanging the others). On CUDA
tensors every exchange first synchronises the device, so the ranks' kernels
(all on one GPU) have finished before their results are read; no kernel ever
waits on another rank.

Test infrastructure only.
"""
from __future__ import annotations

import threading

import torch


class Done:
    """Handle of an already completed asynchronous collective."""

    def wait(self):
        return True


class RankGroup:
    def __init__(self, P: int, timeout: float = 300.0):
        self.P = P
        self.barrier = threading.Barrier(P, timeout=timeout)
        self.local = threading.local()
        self.slots = [None] * P
        self.calls = 0  # collectives completed (rank 0's count)

    # -- torch.distributed surface used by the product
    def get_world_size(self, group=None):
        return self.P

    def get_rank(self, group=None):
        return self.local.rank

    @staticmethod
    def _settle(t):
        if t.is_cuda:
            torch.cuda.synchronize(t.device)

    def _publish(self, item, t):
        self._settle(t)
        self.slots[self.local.rank] = item
        self.barrier.wait()

    def _done(self, t):
        self._settle(t)
        if self.local.rank == 0:
            self.calls += 1
        self.barrier.wait()  # every rank has read the slots

    def all_to_all_single(self, output, input, output_split_sizes=None, input_split_sizes=None,
                          group=None, async_op=False):
        r = self.local.rank
        if input_split_sizes is None:
            self._publish((input, None), input)
            pieces = [self.slots[s][0].reshape(self.P, -1)[r] for s in range(self.P)]
            output.view(self.P, -1).copy_(torch.stack(pieces))
        else:
            self._publish((input.reshape(-1), list(input_split_sizes)), input)
            pieces = []
            for s in range(self.P):
                buf, splits = self.slots[s]
                off = sum(splits[:r])
                pieces.append(buf[off:off + splits[r]])
            want = list(output_split_sizes)
            assert [p.numel() for p in pieces] == want, ([p.numel() for p in pieces], want)
            if pieces:
                output.reshape(-1).copy_(torch.cat([p.to(output.device) for p in pieces]))
        self._done(output)
        return Done() if async_op else None

    def all_gather_into_tensor(self, output, input, group=None, async_op=False):
        self._publish((input, None), input)
        output.view(self.P, -1).copy_(
            torch.stack([self.slots[s][0].reshape(-1) for s in range(self.P)]))
        self._done(output)
        return Done() if async_op else None


def run_ranks(P: int, fake: RankGroup, fn, timeout: float = 600.0):
    """Runs fn(r) on P threads (rank r each); returns the per-rank results
    and raises with every rank's error if any failed."""
    results, errors = [None] * P, []

    def rank(r):
        try:
            fake.local.rank = r
            results[r] = fn(r)
        except BaseException as e:  # noqa: BLE001 -- reported below
            errors.append(f"rank {r}: {type(e).__name__}: {e}")
            fake.barrier.abort()

    threads = [threading.Thread(target=rank, args=(r,)) for r in range(P)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=timeout)
    if any(t.is_alive() for t in threads):
        fake.barrier.abort()
        raise AssertionError("emulated ranks did not finish")
    if errors:
        raise AssertionError("; ".join(errors))
    return results
