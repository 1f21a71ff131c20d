"""Acceptance counters of the verify round, reduced across sequence-sharded ranks.

Each rank owns its own sequences and caches; the only cross-rank exchange of
the path is one int64 vector per round holding the counters the reference
accumulates after every verification (helper/opd_generate.py:551-555):

    accepted_draft  += max(length - 1, 0)   per row
    proposed_draft  += draft_total_token    per row
    accepted_length += length               per row   (avg_acc_length[0])
    verified_rows   += 1                    per row   (avg_acc_length[1])
    finished_rows   += eos flag of the row's packet

On CUDA the increments come from the device packet (`add_device_round`, one
small kernel), and the all_reduce of each round runs on a side stream: it never
sits between two KV kernels, never blocks the host and never orders the next
round's kernels after the other ranks. NCCL (CUDA tensors) and gloo (CPU
tensors) both work; a rank that fails surfaces on the others as an error from
their next `add_round`/`finish` once the process group's timeout expires.
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
    """Job-wide totals of `FIELDS`.

    On CUDA the reduced vectors are accumulated on the device by the side stream (the
    all_reduce's completion is awaited by that stream, never by the host), so rounds do not
    synchronise the ranks' hosts; `finish` reads the totals back once. With CPU tensors
    (gloo) the previous round's reduction is awaited when the next one is queued.
    """

    def __init__(self, device, group=None):
        import torch.distributed as dist
        self.device = torch.device(device)
        self.group = group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.total = torch.zeros(len(FIELDS), dtype=torch.long)
        self._work = None
        self._vec = None
        self._cuda = self.device.type == 'cuda'
        self._stream = torch.cuda.Stream(self.device) if self._cuda else None
        self._total_dev = torch.zeros(len(FIELDS), dtype=torch.long, device=self.device) if self._cuda else None
        # device rounds: a ring of per-round vectors, each reused once the side stream is done with it
        self._ring = [torch.zeros(len(FIELDS), dtype=torch.long, device=self.device) for _ in range(3)] \
            if self._cuda else None
        self._ring_done = [None] * 3
        self._rounds = 0

    def _collect(self):
        if self._work is not None:
            self._work.wait()
            self.total += self._vec
            self._work = None
            self._vec = None

    def add_round(self, values):
        """Queues the reduction of this round's increments."""
        import torch.distributed as dist
        vec = torch.tensor(values, dtype=torch.long)
        if self._cuda:
            vec = vec.pin_memory().to(self.device, non_blocking=True)
            self._stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self._stream):
                vec.record_stream(self._stream)
                if self.distributed:
                    dist.all_reduce(vec, group=self.group, async_op=True).wait()  # the side stream waits
                self._total_dev.add_(vec)
            return
        self._collect()
        if not self.distributed:
            self.total += vec
            return
        self._work = dist.all_reduce(vec, group=self.group, async_op=True)
        self._vec = vec

    def add_device_round(self, packet, batch, proposed_per_row):
        """Queues the reduction of this round's increments, computed on the device from the
        schedule packet (rows [length, eos?, ...]) by one kernel on the current stream; the
        all_reduce and the accumulation run on the side stream. Nothing here waits for the
        other ranks: a ring slot is reused three rounds later, by when its reduction is done."""
        import torch.distributed as dist
        from . import _ops
        slot = self._rounds % len(self._ring)
        self._rounds += 1
        vec = self._ring[slot]
        cur = torch.cuda.current_stream(self.device)
        if self._ring_done[slot] is not None:
            cur.wait_event(self._ring_done[slot])
        _ops.acceptance_counts(packet, batch, proposed_per_row, vec)
        self._stream.wait_stream(cur)
        with torch.cuda.stream(self._stream):
            if self.distributed:
                dist.all_reduce(vec, group=self.group, async_op=True).wait()  # the side stream waits
            self._total_dev.add_(vec)
            done = torch.cuda.Event()
            done.record(self._stream)
        self._ring_done[slot] = done

    def fence(self, stream=None):
        """Orders `stream` (default: the current one) after the reductions queued so far. Call it
        before a kernel that keeps every SM busy (the persistent attention): an all_reduce kernel
        still waiting for a peer rank would otherwise hold SMs that kernel's CTAs wait for."""
        if self._cuda and self.distributed:
            (stream or torch.cuda.current_stream(self.device)).wait_stream(self._stream)

    def finish(self):
        """Waits for the outstanding reductions and returns the totals as a dict."""
        if self._cuda:
            self._stream.synchronize()
            return dict(zip(FIELDS, (self.total + self._total_dev.cpu()).tolist()))
        self._collect()
        return dict(zip(FIELDS, self.total.tolist()))
