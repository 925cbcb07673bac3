"""Device work queue across decode steps.

A serving loop runs the indexer once per decode step over the requests in
flight. Between steps a request's length grows by one token, its block table
gains a page every 64 tokens, and requests are admitted and retired. Shipping
every step's full block table ([B, max_pages] int32: 4 MB for B = 512 at 2048
pages) is wasted work when almost nothing changed, so here:

- the request table (length and block-table row of each request slot) lives
  in device memory for the whole run;
- a step sends one small record: the events since the last step (admit a
  request with its page list, append one page, set a length, retire) and the
  step's batch as a list of slots (int32 words; layout in
  include/dsa_topk_indexer.h, dsa_decode_queue_apply);
- one CUDA graph per batch-size bucket replays [apply the record and gather
  the batch rows (two small kernels), the indexer over the gathered batch]
  with fixed device buffers, so a step is one small host-to-device copy and
  one replay, with no synchronisation between steps.

`RequestTable` is the host's mirror (validation, page bookkeeping, the
record encoder) and needs no GPU; `DecodeQueue` is the device runner.

    dq = DecodeQueue(k_cache, num_slots=512, max_pages=2048, max_batch=512)
    dq.admit(slot=3, seq_len=5000, pages=[...79 page ids...])
    dq.append_page(3, page_id)               # when the request reaches its next page
    topk = dq.step(slots, q, weights)        # lengths += 1, then the indexer
    dq.retire(3)

The reference has no counterpart: its entry point takes a host-built batch
on every call (solution/cuda/kernel.cu:818-887).
"""
import importlib

from ._lib import (DSA_QUEUE_ADMIT, DSA_QUEUE_APPEND_PAGE, DSA_QUEUE_HEADER_WORDS, DSA_QUEUE_RETIRE,
                   DSA_QUEUE_SET_LEN)
from .graph_runner import bucket_for, bucket_sizes

PAGE, TOPK, HEADS, DIM = 64, 2048, 64, 128


class RequestTable:
    """Host mirror of the device request table and encoder of step records.

    Every change is validated here, before it is queued: slots in
    [0, num_slots), admissions only into free slots, pages appended in order
    and at most max_pages per request, and a step only over distinct
    requests in use whose advanced length stays within their pages."""

    def __init__(self, num_slots, max_pages):
        import numpy as np
        if num_slots < 1 or max_pages < 1:
            raise ValueError("num_slots and max_pages must be positive")
        self.np = np
        self.num_slots, self.max_pages = int(num_slots), int(max_pages)
        self.lens = np.full(self.num_slots, -1, dtype=np.int64)  # -1: slot free
        self.npages = np.zeros(self.num_slots, dtype=np.int64)
        self.pages = [[] for _ in range(self.num_slots)]
        self.events = []      # events queued for the next record, each a list of int32 words
        self.event_words = 0  # their total words

    def _queue(self, words):
        self.events.append(words)
        self.event_words += len(words)

    def _slot(self, slot):
        slot = int(slot)
        if not 0 <= slot < self.num_slots:
            raise ValueError(f"slot {slot} outside [0, {self.num_slots})")
        return slot

    def _in_use(self, slot):
        slot = self._slot(slot)
        if self.lens[slot] < 0:
            raise ValueError(f"slot {slot} holds no request")
        return slot

    def admit(self, slot, seq_len, pages):
        slot = self._slot(slot)
        if self.lens[slot] >= 0:
            raise ValueError(f"slot {slot} is in use; retire it first")
        pages = [int(p) for p in pages]
        if len(pages) > self.max_pages:
            raise ValueError(f"{len(pages)} pages exceed max_pages {self.max_pages}")
        if not 0 <= int(seq_len) <= PAGE * len(pages):
            raise ValueError(f"seq_len {seq_len} does not fit {len(pages)} pages")
        pad = (-len(pages)) % 4
        self._queue([DSA_QUEUE_ADMIT, slot, int(seq_len), len(pages)] + pages + [0] * pad)
        self.lens[slot], self.pages[slot], self.npages[slot] = int(seq_len), pages, len(pages)

    def append_page(self, slot, page_id):
        slot = self._in_use(slot)
        idx = len(self.pages[slot])
        if idx >= self.max_pages:
            raise ValueError(f"slot {slot} already holds max_pages {self.max_pages} pages")
        self._queue([DSA_QUEUE_APPEND_PAGE, slot, idx, int(page_id)])
        self.pages[slot].append(int(page_id))
        self.npages[slot] = idx + 1

    def set_len(self, slot, seq_len):
        slot = self._in_use(slot)
        if not 0 <= int(seq_len) <= PAGE * len(self.pages[slot]):
            raise ValueError(f"seq_len {seq_len} does not fit the {len(self.pages[slot])} pages of slot {slot}")
        self._queue([DSA_QUEUE_SET_LEN, slot, int(seq_len), 0])
        self.lens[slot] = int(seq_len)

    def retire(self, slot):
        slot = self._in_use(slot)
        self._queue([DSA_QUEUE_RETIRE, slot, 0, 0])
        self.lens[slot], self.pages[slot], self.npages[slot] = -1, [], 0

    def check_step(self, slots, advance):
        """Raises if the step cannot run; leaves the mirror unchanged.
        Returns the slots as an int64 array."""
        np = self.np
        s = np.asarray(slots, dtype=np.int64).reshape(-1)
        if advance < 0:
            raise ValueError("advance must be >= 0")
        last = getattr(self, "_distinct", None)
        if last is None or last.shape != s.shape or not np.array_equal(last, s):
            # a decode loop usually lists the same slots step after step:
            # range and uniqueness are checked once per distinct list
            if s.size and (s.min() < 0 or s.max() >= self.num_slots):
                raise ValueError(f"a slot lies outside [0, {self.num_slots})")
            if np.unique(s).size != s.size:
                raise ValueError("a slot is listed twice in one step")
            self._distinct = s.copy()
        ln = self.lens[s]
        if (ln < 0).any():
            raise ValueError(f"slot {int(s[np.argmax(ln < 0)])} holds no request")
        over = ln + advance > PAGE * self.npages[s]
        if over.any():
            b = int(np.argmax(over))
            raise ValueError(f"slot {int(s[b])}: length {int(ln[b]) + advance} needs a page it has not been given")
        return s

    def record_words(self, batch):
        """Words of the next record for a batch of `batch` rows."""
        return DSA_QUEUE_HEADER_WORDS + self.event_words + int(batch)

    def take_events(self, max_words):
        """A record with no batch rows that carries the oldest queued events
        fitting in `max_words` words (at least one event), removing them from
        the queue; None when nothing is queued. Lets a burst of changes
        larger than one record go ahead of the step in several records."""
        np = self.np
        if not self.events:
            return None
        n, words = 0, DSA_QUEUE_HEADER_WORDS
        while n < len(self.events) and (n == 0 or words + len(self.events[n]) <= max_words):
            words += len(self.events[n])
            n += 1
        if words > max_words:
            raise ValueError(f"one event of {words - DSA_QUEUE_HEADER_WORDS} words exceeds a record")
        rec = np.empty(words, dtype=np.int32)
        rec[:DSA_QUEUE_HEADER_WORDS] = [words, n, 0, 0, words, 0, 0, 0]
        rec[DSA_QUEUE_HEADER_WORDS:] = [w for ev in self.events[:n] for w in ev]
        self.events = self.events[n:]
        self.event_words -= words - DSA_QUEUE_HEADER_WORDS
        return rec

    def build_record(self, slots, advance=1, checked=False):
        """The step's record (int32 numpy array); applies the advance to the
        mirror and clears the queued events. `checked`: `slots` is the array
        check_step returned for this advance (skips a second check)."""
        np = self.np
        s = slots if checked else self.check_step(slots, advance)
        batch_off = DSA_QUEUE_HEADER_WORDS + self.event_words
        words = batch_off + s.size
        rec = np.empty(words, dtype=np.int32)
        rec[:DSA_QUEUE_HEADER_WORDS] = [words, len(self.events), s.size, int(advance), batch_off, 0, 0, 0]
        if self.events:
            rec[DSA_QUEUE_HEADER_WORDS:batch_off] = [w for ev in self.events for w in ev]
        rec[batch_off:] = s
        self.lens[s] += int(advance)
        self.events, self.event_words = [], 0
        return rec

    def batch_inputs(self, slots):
        """(seq_lens [B], block_table [B, max_pages]) of the listed requests
        as the mirror holds them (zeros past each row's pages), as numpy."""
        np = self.np
        sl = np.array([self.lens[s] for s in slots], dtype=np.int32)
        bt = np.zeros((len(slots), self.max_pages), dtype=np.int32)
        for b, s in enumerate(slots):
            bt[b, :len(self.pages[s])] = self.pages[s]
        return sl, bt


class DecodeQueue:
    """Device runner over a RequestTable (see the module docstring).

    k_cache [num_pages, 64, 1, 132] is the serving system's paged index-K
    cache, fixed for the runner's life (it is captured into the graphs).
    Records are staged through a ring of `ring` pinned host buffers of
    `record_words` int32 words; when the changes queued since the last step
    do not fit in one record with the batch list, the oldest go ahead in
    records of their own (applied outside the graph, on the runner's stream,
    before the step). `step` returns a view of the bucket's output rows,
    valid until the next step that uses the same bucket."""

    def __init__(self, k_cache, num_slots, max_pages, max_batch, record_words=1 << 18, buckets=None, ring=4,
                 stream=None):
        import torch
        self.torch = torch
        self.pkg = importlib.import_module(__package__)
        self.k_cache = k_cache
        self.dev = k_cache.device
        self.table = RequestTable(num_slots, max_pages)
        self.max_pages = int(max_pages)
        self.sizes = list(buckets) if buckets else bucket_sizes(max_batch)
        self.stream = stream or torch.cuda.Stream(self.dev)
        self.record_words = int(record_words)
        if self.record_words < DSA_QUEUE_HEADER_WORDS + max(self.sizes):
            raise ValueError("record_words cannot hold the largest batch list")
        i32 = torch.int32
        self.req_len = torch.full((num_slots,), -1, dtype=i32, device=self.dev)
        self.req_bt = torch.zeros((num_slots, self.max_pages), dtype=i32, device=self.dev)
        self.record = torch.zeros(self.record_words, dtype=i32, device=self.dev)
        self.idle_record = torch.zeros(DSA_QUEUE_HEADER_WORDS, dtype=i32, device=self.dev)  # no events, no rows
        self.idle_record[0] = DSA_QUEUE_HEADER_WORDS
        self.idle_record[4] = DSA_QUEUE_HEADER_WORDS
        self.pinned = [torch.zeros(self.record_words, dtype=i32).pin_memory() for _ in range(int(ring))]
        self.pinned_np = [t.numpy() for t in self.pinned]
        self.copied = [torch.cuda.Event() for _ in range(int(ring))]  # last copy out of each pinned buffer
        self.next_ring = 0
        self.graphs = {}

    # request bookkeeping (queued, sent with the next step's record)
    def append_page(self, slot, page_id):
        self.table.append_page(slot, page_id)

    def set_len(self, slot, seq_len):
        self.table.set_len(slot, seq_len)

    def retire(self, slot):
        self.table.retire(slot)

    def _buffers(self, size):
        torch = self.torch
        return {
            "q": torch.zeros((size, HEADS, DIM), dtype=torch.float8_e4m3fn, device=self.dev),
            "w": torch.zeros((size, HEADS), dtype=torch.float32, device=self.dev),
            "sl": torch.zeros((size,), dtype=torch.int32, device=self.dev),
            "bt": torch.zeros((size, self.max_pages), dtype=torch.int32, device=self.dev),
            "out": torch.empty((size, TOPK), dtype=torch.int32, device=self.dev),
        }

    def _run(self, bufs, record):
        self.pkg.decode_queue_apply(record, self.req_len, self.req_bt, bufs["sl"], bufs["bt"])
        self.pkg.launch_topk_c(bufs["q"], self.k_cache, bufs["w"], bufs["sl"], bufs["bt"], bufs["out"])

    def _capture(self, size):
        torch = self.torch
        bufs = self._buffers(size)
        self.stream.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(self.stream):
            self._run(bufs, self.idle_record)  # warm-up outside capture (library workspaces); changes nothing
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self._run(bufs, self.record)
        self.graphs[size] = (g, bufs)
        return self.graphs[size]

    def input_buffers(self, batch):
        """(q [batch, 64, 128] e4m3, weights [batch, 64] fp32) views of the
        graph buffers a step of `batch` rows reads: a producer that writes
        its outputs there saves step() the two copies."""
        size = bucket_for(batch, self.sizes)
        _, bufs = self.graphs.get(size) or self._capture(size)
        return bufs["q"][:batch], bufs["w"][:batch]

    def step(self, slots, q, weights, advance=1):
        """One decode step over the requests in `slots` (batch order): their
        lengths grow by `advance`, then the indexer runs with q [B, 64, 128]
        e4m3 and weights [B, 64] fp32 (device or pinned host tensors, or the
        views input_buffers(B) returned, which are used in place).
        Returns the [B, 2048] top-K slots (a view, see the class docstring)."""
        torch = self.torch
        B = len(slots)
        if B == 0:
            raise ValueError("empty step")
        if tuple(q.shape) != (B, HEADS, DIM) or tuple(weights.shape) != (B, HEADS):
            raise ValueError("q must be [B, 64, 128] and weights [B, 64] for the B listed slots")
        size = bucket_for(B, self.sizes)
        s = self.table.check_step(slots, advance)
        g, bufs = self.graphs.get(size) or self._capture(size)
        cur = torch.cuda.current_stream(self.dev)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            while self.table.record_words(B) > self.record_words:  # a burst of changes: send the oldest first
                rec = self.table.take_events(self.record_words)
                self._send(rec)
                self.pkg.decode_queue_apply(self.record, self.req_len, self.req_bt, bufs["sl"], bufs["bt"])
            self._send(self.table.build_record(s, advance, checked=True))
            if q.data_ptr() != bufs["q"].data_ptr():
                bufs["q"][:B].copy_(q, non_blocking=True)
            if weights.data_ptr() != bufs["w"].data_ptr():
                bufs["w"][:B].copy_(weights, non_blocking=True)
            g.replay()
        cur.wait_stream(self.stream)
        return bufs["out"][:B]

    def _send(self, rec):
        """Copies one record into the device record buffer (on the current
        stream) through the next pinned ring buffer."""
        n = rec.size
        j = self.next_ring
        self.next_ring = (j + 1) % len(self.pinned)
        self.copied[j].synchronize()  # the copy that last read this pinned buffer has finished
        self.pinned_np[j][:n] = rec
        self.record[:n].copy_(self.pinned[j][:n], non_blocking=True)
        self.copied[j].record(self.torch.cuda.current_stream(self.dev))

    def admit(self, slot, seq_len, pages):
        pages = list(pages)
        if DSA_QUEUE_HEADER_WORDS + 4 + len(pages) + 3 > self.record_words:
            raise ValueError(f"an admission of {len(pages)} pages does not fit a record of {self.record_words} words")
        self.table.admit(slot, seq_len, pages)

    def device_table(self):
        """(req_len, req_block_table) as the device holds them (synchronises)."""
        self.torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        return self.req_len.cpu(), self.req_bt.cpu()
