"""Decode-loop runners: the indexer call (GraphRunner), or the indexer and
the sparse attention over its output (DecodeStepRunner), captured once per
batch-size bucket into a CUDA graph with fixed device buffers, replayed
every step.

A serving loop calls the indexer once per decode step with a different
batch (requests come and go) against the same paged K cache. Launch cost
then matters at the sizes of config 1 (tens of microseconds per call), so
the call is recorded into a CUDA graph per bucket of batch sizes (powers of
two by default) and per block-table width, with the K cache fixed at
capture. A step copies q, weights, seq_lens and block_table into the
bucket's buffers (padding rows get seq_len 0: all -1, discarded), replays
the graph and returns a view of the first B output rows.

The workspace the library keeps per stream is created by the warm-up call
before capture, so a replay allocates nothing.
"""
import importlib

PAGE, TOPK, HEADS, DIM = 64, 2048, 64, 128


def bucket_sizes(max_batch, smallest=1):
    """Powers of two from `smallest` up to the first one >= max_batch."""
    out, b = [], max(1, int(smallest))
    while True:
        out.append(b)
        if b >= max_batch:
            return out
        b *= 2


def bucket_for(batch, sizes):
    """The smallest bucket that holds `batch` rows."""
    for s in sizes:
        if batch <= s:
            return s
    raise ValueError(f"batch {batch} exceeds the largest bucket {sizes[-1]}")


class GraphRunner:
    """runner = GraphRunner(k_cache, max_batch=64, max_pages=512)
    topk = runner(q, weights, seq_lens, block_table)   # [B, 2048] int32 view

    k_cache: the serving system's paged cache ([num_pages, 64, 1, 132]);
    inputs of a step may be on the host (pinned) or the device; their
    block_table may be narrower than max_pages (the rest reads as page 0 and
    is never used: only pages below a row's seq_len are read)."""

    def __init__(self, k_cache, max_batch, max_pages, buckets=None, stream=None):
        import torch
        self.torch = torch
        self.pkg = importlib.import_module(__package__)
        self.k_cache = k_cache
        self.dev = k_cache.device
        self.max_pages = int(max_pages)
        self.sizes = list(buckets) if buckets else bucket_sizes(max_batch)
        self.stream = stream or torch.cuda.Stream(self.dev)
        self.graphs = {}

    def _buffers(self, size):
        torch = self.torch
        return {
            "q": torch.zeros((size, HEADS, DIM), dtype=torch.float8_e4m3fn, device=self.dev),
            "w": torch.zeros((size, HEADS), dtype=torch.float32, device=self.dev),
            "sl": torch.zeros((size,), dtype=torch.int32, device=self.dev),
            "bt": torch.zeros((size, self.max_pages), dtype=torch.int32, device=self.dev),
            "out": torch.empty((size, TOPK), dtype=torch.int32, device=self.dev),
        }

    def _step(self, bufs):
        self.pkg.launch_topk_c(bufs["q"], self.k_cache, bufs["w"], bufs["sl"], bufs["bt"], bufs["out"])

    def _capture(self, size):
        torch = self.torch
        bufs = self._buffers(size)
        self.stream.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(self.stream):
            self._step(bufs)  # warm-up outside capture: creates the library's per-stream workspaces
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self._step(bufs)
        self.graphs[size] = (g, bufs)
        return self.graphs[size]

    def _stage(self, q, weights, seq_lens, block_table):
        """Copies a step's indexer inputs into its bucket's buffers."""
        B = int(q.shape[0])
        if block_table.shape[1] > self.max_pages:
            raise ValueError(f"block_table has {block_table.shape[1]} columns, the runner holds {self.max_pages}")
        size = bucket_for(B, self.sizes)
        g, bufs = self.graphs.get(size) or self._capture(size)
        bufs["q"][:B].copy_(q, non_blocking=True)
        bufs["w"][:B].copy_(weights, non_blocking=True)
        bufs["sl"][:B].copy_(seq_lens, non_blocking=True)
        bufs["sl"][B:].zero_()
        bufs["bt"][:B, :block_table.shape[1]].copy_(block_table, non_blocking=True)
        return B, g, bufs

    def _replay(self, g):
        cur = self.torch.cuda.current_stream(self.dev)
        self.stream.wait_stream(cur)
        g.replay()
        cur.wait_stream(self.stream)

    def __call__(self, q, weights, seq_lens, block_table):
        B, g, bufs = self._stage(q, weights, seq_lens, block_table)
        self._replay(g)
        return bufs["out"][:B]


class DecodeStepRunner(GraphRunner):
    """The indexer and the sparse attention over its output in one CUDA graph
    per bucket (one replay per decode step):

        runner = DecodeStepRunner(k_cache, ckv_cache, kpe_cache, sm_scale, max_batch=64, max_pages=512)
        topk, out, lse = runner(q, weights, seq_lens, block_table, q_nope, q_pe)

    ckv_cache [pages, 64, 512] / kpe_cache [pages, 64, 64] (bf16) are the
    attention's page pools, addressed by the same physical slots the indexer
    emits; q_nope [B, 16, 512] / q_pe [B, 16, 64] bf16. Padding rows have no
    slots (zero output, lse -inf) and are not returned."""

    def __init__(self, k_cache, ckv_cache, kpe_cache, sm_scale, max_batch, max_pages, buckets=None, stream=None):
        super().__init__(k_cache, max_batch, max_pages, buckets, stream)
        self.ckv, self.kpe, self.sm_scale = ckv_cache, kpe_cache, float(sm_scale)

    def _buffers(self, size):
        torch = self.torch
        bufs = super()._buffers(size)
        bufs.update({
            "qn": torch.zeros((size, 16, 512), dtype=torch.bfloat16, device=self.dev),
            "qp": torch.zeros((size, 16, 64), dtype=torch.bfloat16, device=self.dev),
            "ao": torch.empty((size, 16, 512), dtype=torch.bfloat16, device=self.dev),
            "lse": torch.empty((size, 16), dtype=torch.float32, device=self.dev),
        })
        return bufs

    def _step(self, bufs):
        super()._step(bufs)
        self.pkg.sparse_attention(bufs["qn"], bufs["qp"], self.ckv, self.kpe, bufs["out"], self.sm_scale,
                                  output=bufs["ao"], lse=bufs["lse"])

    def __call__(self, q, weights, seq_lens, block_table, q_nope, q_pe):
        B, g, bufs = self._stage(q, weights, seq_lens, block_table)
        bufs["qn"][:B].copy_(q_nope, non_blocking=True)
        bufs["qp"][:B].copy_(q_pe, non_blocking=True)
        self._replay(g)
        return bufs["out"][:B], bufs["ao"][:B], bufs["lse"][:B]
