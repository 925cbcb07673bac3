"""Device work queue across decode steps: the host mirror and record encoder
(CPU), and the device runner against direct indexer calls on host-built
batches (GPU, bit for bit), including malformed records."""
import numpy as np
import pytest
import torch

from conftest import package, workloads


def _mod():
    return __import__("importlib").import_module(package().__name__ + ".decode_queue")


def _lib():
    return package()._lib


def apply_model(rec, req_len, req_bt, capacity):
    """Test-side restatement of the two device kernels (decode_queue.cuh):
    returns (seq_lens [capacity], block-table rows {b: pages}, bad) and
    updates req_len / req_bt in place."""
    L = _lib()
    H = L.DSA_QUEUE_HEADER_WORDS
    S, mp = req_bt.shape
    words, n_ev, B, adv, boff = rec[:5]
    sl = np.zeros(capacity, dtype=np.int64)
    rows = {}
    if not (H <= words <= len(rec) and n_ev >= 0 and 0 <= B <= capacity and adv >= 0 and boff >= H
            and boff + B <= words):
        return sl, rows, True
    bad = False
    off = H
    for _ in range(n_ev):
        if off + 4 > boff:
            bad = True
            break  # the apply kernel stops; the gather still runs
        t, s, a, b = rec[off:off + 4]
        off += 4
        ok = 0 <= s < S
        if t == L.DSA_QUEUE_ADMIT:
            pw = (b + 3) // 4 * 4
            if b < 0 or b > mp or off + pw > boff:
                bad = True
                break
            if ok and a >= 0:
                req_bt[s, :b] = rec[off:off + b]
                req_len[s] = a
            else:
                bad = True
            off += pw
        elif t == L.DSA_QUEUE_APPEND_PAGE:
            if ok and 0 <= a < mp:
                req_bt[s, a] = b
            else:
                bad = True
        elif t == L.DSA_QUEUE_SET_LEN:
            if ok and a >= 0:
                req_len[s] = a
            else:
                bad = True
        elif t == L.DSA_QUEUE_RETIRE:
            if ok:
                req_len[s] = -1
            else:
                bad = True
        else:
            bad = True
            break
    for b in range(B):
        s = rec[boff + b]
        if not (0 <= s < S) or req_len[s] < 0:
            bad = True
            continue
        req_len[s] += adv
        sl[b] = req_len[s]
        rows[b] = req_bt[s, :min((sl[b] + 63) // 64, mp)].copy()
    return sl, rows, bad


def _script(table, rng, free_pages, steps, max_batch):
    """Random admissions, page appends, length changes and retirements with
    a decode step after each round; yields (record, slots)."""
    active = []
    for _ in range(steps):
        for _ in range(int(rng.integers(0, 3))):
            free = [s for s in range(table.num_slots) if table.lens[s] < 0]
            if not free:
                break
            s = int(rng.choice(free))
            n = int(rng.integers(1, 9))
            pages = [free_pages.pop() for _ in range(n)]
            table.admit(s, int(rng.integers(0, 64 * n - 3)), pages)
            active.append(s)
        if active and rng.random() < 0.3:
            s = active.pop(int(rng.integers(0, len(active))))
            free_pages += table.pages[s]
            table.retire(s)
        if active and rng.random() < 0.2:
            s = int(rng.choice(active))
            table.set_len(s, int(rng.integers(0, 64 * len(table.pages[s]) - 3)))
        for s in active:  # give every request room for the next token
            if table.lens[s] + 1 > 64 * len(table.pages[s]) and len(table.pages[s]) < table.max_pages:
                table.append_page(s, free_pages.pop())
        slots = [s for s in active if table.lens[s] + 1 <= 64 * len(table.pages[s])]
        rng.shuffle(slots)
        slots = slots[:max_batch]
        if not slots:
            continue
        yield table.build_record(slots, 1), slots


def test_record_encoding_matches_model():
    """Records built by RequestTable, applied by the restatement of the
    device kernels, reproduce the mirror's lengths and block tables."""
    m = _mod()
    t = m.RequestTable(num_slots=12, max_pages=10)
    req_len = np.full(12, -1, dtype=np.int64)
    req_bt = np.zeros((12, 10), dtype=np.int64)
    rng = np.random.default_rng(3)
    n_steps = 0
    for rec, slots in _script(t, rng, list(range(3000)), 60, 8):
        sl, rows, bad = apply_model([int(x) for x in rec], req_len, req_bt, 8)
        assert not bad
        ref_sl, ref_bt = t.batch_inputs(slots)
        assert list(sl[:len(slots)]) == list(ref_sl) and not sl[len(slots):].any()
        for b in range(len(slots)):
            assert list(rows[b]) == list(ref_bt[b, :len(rows[b])])
        for s in range(12):
            assert req_len[s] == t.lens[s]
            assert list(req_bt[s, :len(t.pages[s])]) == t.pages[s]
        n_steps += 1
    assert n_steps > 30


def test_event_bursts_split_into_records():
    """Queued changes larger than one record go out as batch-less records of
    whole events (oldest first), then the step's record; applied in order
    they give the same table as one large record."""
    m = _mod()
    t = m.RequestTable(num_slots=8, max_pages=40)
    req_len = np.full(8, -1, dtype=np.int64)
    req_bt = np.zeros((8, 40), dtype=np.int64)
    for s in range(6):
        t.admit(s, 64 * (5 + s) - 7, list(range(100 * s, 100 * s + 5 + s)))
    t.retire(2)
    t.append_page(3, 999)
    cap = 48
    recs = []
    while t.record_words(4) > cap:
        r = t.take_events(cap)
        assert r[2] == 0 and len(r) <= cap
        recs.append(r)
    recs.append(t.build_record([0, 1, 3, 5], 1))
    assert len(recs) > 2 and len(recs[-1]) <= cap and t.events == []
    for r in recs:
        sl, rows, bad = apply_model([int(x) for x in r], req_len, req_bt, 4)
        assert not bad
    ref_sl, ref_bt = t.batch_inputs([0, 1, 3, 5])
    assert list(sl) == list(ref_sl)
    for b in range(4):
        assert list(rows[b]) == list(ref_bt[b, :len(rows[b])])
    for s in range(8):
        assert req_len[s] == t.lens[s]
    with pytest.raises(ValueError):
        t.admit(6, 10, list(range(40)))
        t.take_events(20)  # one admission of 40 pages cannot fit 20 words


def test_request_table_rejects_bad_changes():
    m = _mod()
    t = m.RequestTable(num_slots=4, max_pages=3)
    with pytest.raises(ValueError):
        t.admit(4, 10, [1])                 # slot out of range
    with pytest.raises(ValueError):
        t.admit(0, 200, [1, 2, 3])          # longer than its pages
    with pytest.raises(ValueError):
        t.admit(0, 10, [1, 2, 3, 4])        # more than max_pages
    t.admit(0, 64, [7])
    with pytest.raises(ValueError):
        t.admit(0, 1, [8])                  # slot in use
    with pytest.raises(ValueError):
        t.build_record([0], 1)              # needs a second page first
    with pytest.raises(ValueError):
        t.build_record([0, 0], 0)           # listed twice
    with pytest.raises(ValueError):
        t.build_record([1], 0)              # free slot
    t.append_page(0, 9)
    t.append_page(0, 10)
    with pytest.raises(ValueError):
        t.append_page(0, 11)                # past max_pages
    rec = t.build_record([0], 1)
    assert rec[1] == 3 and rec[2] == 1 and rec[rec[4]] == 0 and len(rec) == rec[0]  # admit + two appends
    assert t.lens[0] == 65
    t.retire(0)
    with pytest.raises(ValueError):
        t.set_len(0, 1)


# ---------------------------------------------------------------- GPU


def _queue_setup(n_pages=2000, seed=11):
    """A K pool of n_pages pages, every page written (benchmark distributions)."""
    W = workloads()
    kc = torch.zeros((n_pages, 64, 1, 132), dtype=torch.uint8, device="cuda")
    W.write_pages(kc, torch.arange(n_pages), W._gen(seed, "cuda"))
    return kc


@pytest.mark.gpu
def test_queue_steps_equal_direct_calls():
    """A decode loop through DecodeQueue (records, device table, one graph
    per bucket) gives bit for bit what launch_topk_c gives on the batch the
    host mirror describes, step after step; the device table ends equal to
    the mirror."""
    pkg = package()
    m = _mod()
    kc = _queue_setup()
    dq = m.DecodeQueue(kc, num_slots=24, max_pages=40, max_batch=16, buckets=[4, 16])
    rng = np.random.default_rng(5)
    free = list(range(kc.shape[0]))
    rng.shuffle(free)
    free = [int(p) for p in free]
    g = torch.Generator(device="cuda").manual_seed(9)
    steps = 0
    pkg.device_status(0, clear=True)
    table = dq.table
    active = []
    for it in range(40):
        for _ in range(int(rng.integers(0, 3))):
            cand = [s for s in range(24) if table.lens[s] < 0]
            if not cand:
                break
            s = int(rng.choice(cand))
            n = int(rng.integers(1, 30))
            dq.admit(s, int(rng.integers(0, 64 * n - 1)), [free.pop() for _ in range(n)])
            active.append(s)
        if active and rng.random() < 0.25:
            s = active.pop(int(rng.integers(0, len(active))))
            free += table.pages[s]
            dq.retire(s)
        for s in active:
            if table.lens[s] + 1 > 64 * len(table.pages[s]) and len(table.pages[s]) < 40:
                dq.append_page(s, free.pop())
        slots = [s for s in active if table.lens[s] + 1 <= 64 * len(table.pages[s])]
        rng.shuffle(slots)
        slots = slots[:16]
        if not slots:
            continue
        B = len(slots)
        q = (torch.randn((B, 64, 128), generator=g, device="cuda") * 0.5).to(torch.float8_e4m3fn)
        w = torch.rand((B, 64), generator=g, device="cuda") / 8
        if it % 2:
            got = dq.step(slots, q, w).clone()
        else:  # the producer writes straight into the graph's input buffers
            qb, wb = dq.input_buffers(B)
            qb.copy_(q)
            wb.copy_(w)
            got = dq.step(slots, qb, wb).clone()
        sl, bt = table.batch_inputs(slots)  # the mirror after this step's advance
        ref = torch.empty((B, 2048), dtype=torch.int32, device="cuda")
        pkg.launch_topk_c(q, kc, w, torch.from_numpy(sl).cuda(), torch.from_numpy(bt).cuda(), ref)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (it, B)
        steps += 1
    assert steps > 25 and set(dq.graphs) == {4, 16}
    assert pkg.device_status(0) == 0
    req_len, req_bt = dq.device_table()
    for s in range(24):
        assert int(req_len[s]) == table.lens[s]
        assert req_bt[s, :len(table.pages[s])].tolist() == table.pages[s]


@pytest.mark.gpu
def test_queue_bursts_larger_than_a_record():
    """Admissions of many pages with a small record buffer: the queue sends
    them in several records before the step; results equal direct calls."""
    pkg = package()
    m = _mod()
    kc = _queue_setup(n_pages=400, seed=12)
    dq = m.DecodeQueue(kc, num_slots=8, max_pages=64, max_batch=8, buckets=[8], record_words=96)
    g = torch.Generator(device="cuda").manual_seed(4)
    pages = torch.randperm(400, generator=torch.Generator().manual_seed(3)).tolist()
    for s in range(8):
        n = 20 + 5 * s
        dq.admit(s, 64 * n - 3 * s - 1, pages[:n])
        pages = pages[n:]
    for step in range(3):
        slots = [7, 0, 3, 5, 1] if step != 1 else [2, 4, 6]
        B = len(slots)
        q = (torch.randn((B, 64, 128), generator=g, device="cuda") * 0.5).to(torch.float8_e4m3fn)
        w = torch.rand((B, 64), generator=g, device="cuda") / 8
        got = dq.step(slots, q, w, advance=0).clone()
        sl, bt = dq.table.batch_inputs(slots)
        ref = torch.empty((B, 2048), dtype=torch.int32, device="cuda")
        pkg.launch_topk_c(q, kc, w, torch.from_numpy(sl).cuda(), torch.from_numpy(bt).cuda(), ref)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), step
    assert pkg.device_status(0) == 0


@pytest.mark.gpu
def test_malformed_records_flag_and_skip():
    """Events and rows naming bad slots or page indices are skipped with
    DSA_STATUS_BAD_RECORD; the valid ones still apply; a record whose header
    does not fit is dropped whole (every row empty). No fault."""
    pkg = package()
    L = _lib()
    H = L.DSA_QUEUE_HEADER_WORDS
    S, mp, C = 6, 8, 4
    req_len = torch.full((S,), -1, dtype=torch.int32, device="cuda")
    req_bt = torch.zeros((S, mp), dtype=torch.int32, device="cuda")
    sl = torch.full((C,), 7, dtype=torch.int32, device="cuda")
    bt = torch.zeros((C, mp), dtype=torch.int32, device="cuda")
    ev = [L.DSA_QUEUE_ADMIT, 2, 100, 2, 11, 12, 0, 0,       # good: slot 2, 100 keys on pages 11, 12
          L.DSA_QUEUE_APPEND_PAGE, 2, 9, 5,                 # page index 9 >= max_pages: skipped
          L.DSA_QUEUE_SET_LEN, 7, 5, 0,                     # slot 7 >= num_slots: skipped
          L.DSA_QUEUE_ADMIT, 4, 10, 1, 30, 0, 0, 0]         # good: slot 4
    batch = [2, 5, 4]                                       # slot 5 is free: an empty row
    boff = H + len(ev)
    rec = [boff + len(batch), 4, len(batch), 1, boff, 0, 0, 0] + ev + batch
    pkg.device_status(0, clear=True)
    pkg.decode_queue_apply(torch.tensor(rec, dtype=torch.int32, device="cuda"), req_len, req_bt, sl, bt)
    torch.cuda.synchronize()
    assert pkg.device_status(0, clear=True) & pkg.DSA_STATUS_BAD_RECORD
    assert sl.tolist() == [101, 0, 11, 0]
    assert bt[0, :2].tolist() == [11, 12] and bt[2, 0].item() == 30
    assert req_len.tolist() == [-1, -1, 101, -1, 11, -1]
    # unknown event type: the rest of the record is not applied, the batch still gathers
    rec2 = [H + 4 + 1, 1, 1, 0, H + 4, 0, 0, 0] + [99, 2, 0, 0] + [2]
    pkg.decode_queue_apply(torch.tensor(rec2, dtype=torch.int32, device="cuda"), req_len, req_bt, sl, bt)
    torch.cuda.synchronize()
    assert pkg.device_status(0, clear=True) & pkg.DSA_STATUS_BAD_RECORD
    assert sl.tolist() == [101, 0, 0, 0]
    # header claims more words than the record holds: dropped, every row empty
    rec3 = [10 ** 6, 0, 1, 1, H, 0, 0, 0, 2]
    pkg.decode_queue_apply(torch.tensor(rec3, dtype=torch.int32, device="cuda"), req_len, req_bt, sl, bt)
    torch.cuda.synchronize()
    assert pkg.device_status(0, clear=True) & pkg.DSA_STATUS_BAD_RECORD
    assert sl.tolist() == [0, 0, 0, 0] and req_len.tolist() == [-1, -1, 101, -1, 11, -1]
