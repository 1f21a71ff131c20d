"""Acceptance counters of the verify round, reduced across sequence-sharded ranks.

Each rank owns its own sequences and caches; the only cross-rank exchange of
the path is one int64 vector per round holding the counters the reference
accumulates after every verification (helper/opd_generate.py:551-555):

    accepted_draft  += max(length - 1, 0)   per row
    proposed_draft  += draft_total_token    per row
    accepted_length += length               per row   (avg_acc_length[0])
    verified_rows   += 1                    per row   (avg_acc_length[1])
    finished_rows   += eos flag of the row's packet

The all_reduce of round i is issued on a side stream and waited for at round
i + 1, so it never sits between two KV kernels. NCCL (CUDA tensors) and gloo
(CPU tensors) both work; a rank that fails surfaces on the others as an error
from their next `add_round`/`finish` once the process group's timeout expires.
"""
import torch

FIELDS = ('accepted_draft', 'proposed_draft', 'accepted_length', 'verified_rows', 'finished_rows')


def round_increments(rows, proposed_per_row):
    """Counter increments of one round from the host packet rows `[length, eos?, ...]`."""
    return [sum(max(int(r[0]) - 1, 0) for r in rows),
            proposed_per_row * len(rows),
            sum(int(r[0]) for r in rows),
            len(rows),
            sum(1 for r in rows if r[1])]


class AcceptanceCounters:
    """Job-wide totals of `FIELDS`; `total` holds every reduction that has completed."""

    def __init__(self, device, group=None):
        import torch.distributed as dist
        self.device = torch.device(device)
        self.group = group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.total = torch.zeros(len(FIELDS), dtype=torch.long)
        self._work = None
        self._vec = None
        self._stream = torch.cuda.Stream(self.device) if self.device.type == 'cuda' and self.distributed else None

    def _collect(self):
        if self._work is not None:
            self._work.wait()
            if self._stream is not None:
                torch.cuda.current_stream(self.device).wait_stream(self._stream)
            self.total += self._vec.cpu()
            self._work = None
            self._vec = None

    def add_round(self, values):
        """Queues the reduction of this round's increments and folds in the previous round's."""
        import torch.distributed as dist
        self._collect()
        vec = torch.tensor(values, dtype=torch.long)
        if not self.distributed:
            self.total += vec
            return
        if self._stream is not None:
            vec = vec.pin_memory().to(self.device, non_blocking=True)
            self._stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self._stream):
                vec.record_stream(self._stream)
                self._work = dist.all_reduce(vec, group=self.group, async_op=True)
        else:
            self._work = dist.all_reduce(vec, group=self.group, async_op=True)
        self._vec = vec

    def finish(self):
        """Waits for the outstanding reduction and returns the totals as a dict."""
        self._collect()
        return dict(zip(FIELDS, self.total.tolist()))
