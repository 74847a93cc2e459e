"""Device-side KV bookkeeping against the reference's KvCache rules.

DevicePages (lstk_cuda_kv_alloc / lstk_cuda_kv_release) must hand out exactly the cells,
positions and blocks that sequential KvCache::alloc(seq, n) calls give (src/kv_cache.cpp:59-83),
and free blocks in the order truncate_seq / remove_seq push them (src/kv_cache.cpp:85-132). A
random serving trace (steps of prompt chunks and decode tokens over a changing set of slots,
prefix-reuse truncations, removals, a cache that runs full) runs on both; after every operation the free stack, block tables, lengths and
high-water mark must be identical.
"""
import numpy as np
import pytest
import torch

import localstack_b200 as L
from localstack_b200.kv_cache import KvCache
from localstack_b200.pages import DevicePages

pytestmark = pytest.mark.gpu


def _compare(kv, dp, n_slots, max_blocks, tag):
    assert np.array_equal(dp.free_list(), kv.free_blocks()), tag
    lens = dp.seq_lens.cpu().numpy()
    bt = dp.block_tables.cpu().numpy()
    for s in range(n_slots):
        assert lens[s] == kv.length(s), (tag, s)
        blocks = kv.seq_blocks(s)
        assert np.array_equal(bt[s, : blocks.size].view(np.uint32), blocks), (tag, s)
    assert int(dp.used_hwm.item()) == kv.used_hwm, tag


def _host_alloc(kv, slots, counts):
    """Sequential KvCache::alloc calls: (cells, positions, ok) laid out like DevicePages.alloc."""
    cells, pos, ok = [], [], []
    for s, c in zip(slots, counts):
        r = kv.alloc(int(s), int(c))
        ok.append(1 if r is not None else 0)
        cells.append(r[0] if r is not None else np.full(c, -1, np.int64))
        pos.append(r[1] if r is not None else np.full(c, -1, np.int32))
    return np.concatenate(cells + [np.zeros(0, np.int64)]), np.concatenate(pos + [np.zeros(0, np.int32)]), ok


@pytest.mark.parametrize("n_slots,size,seed", [(64, 4096, 0), (1500, 65536, 1), (200, 2048, 2), (2048, 32768, 3)])
def test_trace_matches_kv_cache(n_slots, size, seed):
    """Continuous-batching steps (prompt chunks mixed with decode tokens), prefix-reuse truncations
    and removals; the cache runs full in the small cases, so some requests fail mid-step."""
    rng = np.random.default_rng(seed)
    max_blocks = size // 32
    perm = rng.permutation(size // 32).astype(np.uint32)
    kv = KvCache(size)
    kv.set_free_blocks(perm)
    dp = DevicePages(size, n_slots, max_blocks, free_blocks=perm)
    for it in range(60):
        op = rng.random()
        if op < 0.75:
            k = int(rng.integers(1, n_slots + 1))
            slots = rng.choice(n_slots, k, replace=False).astype(np.int32)
            for _ in range(int(rng.integers(1, 20))):  # several steps over the same batch
                counts = np.where(rng.random(k) < 0.9, 1, rng.integers(0, 300, k)).astype(np.int32)
                total = int(counts.sum())
                cells, pos, ok = dp.alloc(torch.from_numpy(slots).cuda(), torch.from_numpy(counts).cuda(), total)
                want_c, want_p, want_ok = _host_alloc(kv, slots, counts)
                L.check_status()
                assert np.array_equal(ok.cpu().numpy(), want_ok), it
                assert np.array_equal(cells.cpu().numpy(), want_c), it
                assert np.array_equal(pos.cpu().numpy(), want_p), it
        else:
            s = int(rng.integers(0, n_slots))
            keep = 0 if op < 0.85 else int(rng.integers(0, max(1, kv.length(s)) + 40))
            dp.release(s, keep)
            if keep > 0:
                kv.truncate_seq(s, keep)
            else:
                kv.remove_seq(s)
        _compare(kv, dp, n_slots, max_blocks, it)


def test_failed_request_takes_nothing_and_later_ones_fit():
    kv = KvCache(256)  # 8 blocks
    dp = DevicePages(256, 4, 8)
    slots = torch.tensor([0, 1, 2, 3], dtype=torch.int32, device="cuda")
    counts = np.array([100, 200, 64, 1], np.int32)  # 4 blocks, 7 (fails: 4 left), 2, 1
    cells, pos, ok = dp.alloc(slots, torch.from_numpy(counts).cuda(), int(counts.sum()))
    want_c, want_p, want_ok = _host_alloc(kv, [0, 1, 2, 3], counts)
    assert want_ok == [1, 0, 1, 1]
    assert ok.cpu().tolist() == want_ok
    assert np.array_equal(cells.cpu().numpy(), want_c) and np.array_equal(pos.cpu().numpy(), want_p)
    _compare(kv, dp, 4, 8, "fail")
    # outputs too short for the counts: nothing is allocated and the device status says so
    before = (dp.free_list(), dp.seq_lens.clone(), dp.block_tables.clone())
    _, _, ok = dp.alloc(slots, torch.from_numpy(counts).cuda(), 10)
    with pytest.raises(L.LstkError):
        L.check_status()
    assert ok.cpu().tolist() == [0, 0, 0, 0]
    assert np.array_equal(dp.free_list(), before[0]) and torch.equal(dp.seq_lens, before[1])
    assert torch.equal(dp.block_tables, before[2])


def test_invalid_items_write_no_outputs():
    """Items with an out-of-range slot or a negative count reserve no output entries and write
    none: the valid slots after them keep their cells and positions, the entries past the valid
    tokens stay untouched, and the device status reports the bad item."""
    kv = KvCache(1024)
    dp = DevicePages(1024, 4, 32)
    dev = "cuda"
    for slots_l, counts_l in (([7, 1, -3, 2], [5, 3, 4, 2]), ([0, 1, 3], [-2, 40, 1])):
        slots = torch.tensor(slots_l, dtype=torch.int32, device=dev)
        counts = torch.tensor(counts_l, dtype=torch.int32, device=dev)
        cells = torch.full((64,), -7, dtype=torch.int64, device=dev)
        pos = torch.full((64,), -7, dtype=torch.int32, device=dev)
        _, _, ok = dp.alloc(slots, counts, 64, cells=cells, positions=pos)
        with pytest.raises(L.LstkError) as e:
            L.check_status()
        assert e.value.code == -6  # LSTK_ERR_DEVICE_INDEX
        valid = [(s, c) for s, c in zip(slots_l, counts_l) if 0 <= s < 4 and c >= 0]
        want_c, want_p, _ = _host_alloc(kv, [s for s, _ in valid], [c for _, c in valid])
        n = want_c.size
        assert ok.cpu().tolist() == [1 if (0 <= s < 4 and c >= 0) else 0 for s, c in zip(slots_l, counts_l)]
        assert np.array_equal(cells[:n].cpu().numpy(), want_c) and np.array_equal(pos[:n].cpu().numpy(), want_p)
        assert bool((cells[n:] == -7).all()) and bool((pos[n:] == -7).all())
        _compare(kv, dp, 4, 32, "invalid items")


def test_full_cache_and_full_table():
    # 4 blocks for 3 slots of at most 2 blocks: the stack runs empty mid-step; a full table row fails
    kv = KvCache(128)
    dp = DevicePages(128, 3, 2)
    slots = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    for step in range(70):
        cells, pos, ok = dp.alloc_step(slots)
        ok = ok.cpu().numpy()
        for i, s in enumerate([0, 1, 2]):
            table_full = kv.length(s) == 64
            r = None if table_full else kv.alloc(s, 1)
            assert ok[i] == (1 if r is not None else 0), (step, s)
            if r is not None:
                assert int(cells[i]) == r[0][0] and int(pos[i]) == r[1][0]
    assert kv.n_free_cells() == 0
    _compare(kv, dp, 3, 2, "full")


def test_decode_step_stays_on_device():
    # allocate -> append -> decode with the device tables, against the same steps on host tables
    Hq, Hkv, size, n_slots = 16, 8, 4096, 8
    dev = "cuda"
    rng = np.random.default_rng(5)
    kv = KvCache(size)
    dp = DevicePages(size, n_slots, size // 32)
    kc, vc = L.alloc_cache(size, Hkv, dev), L.alloc_cache(size, Hkv, dev)
    kc2, vc2 = L.alloc_cache(size, Hkv, dev), L.alloc_cache(size, Hkv, dev)
    rope = L.rope_table(4096, dev)
    slots = torch.arange(n_slots, dtype=torch.int32, device=dev)
    for step in range(70):
        q = torch.randn(n_slots, Hq, 128, device=dev)
        k = torch.randn(n_slots, Hkv, 128, device=dev)
        v = torch.randn(n_slots, Hkv, 128, device=dev)
        cells, pos, _ = dp.alloc_step(slots)
        qr = L.kv_append(kc, vc, q, k, v, pos, cells, rope)
        out = L.attn_decode(kc, vc, qr, dp.block_tables, dp.seq_lens)
        hc, hp = zip(*[kv.alloc(s, 1) for s in range(n_slots)])
        hc = torch.from_numpy(np.concatenate(hc)).to(dev)
        hp = torch.from_numpy(np.concatenate(hp)).to(dev)
        qr2 = L.kv_append(kc2, vc2, q, k, v, hp, hc, rope)
        bt, lens = kv.block_tables(np.arange(n_slots, dtype=np.int32), size // 32)
        out2 = L.attn_decode(kc2, vc2, qr2, torch.from_numpy(bt).to(dev), torch.from_numpy(lens).to(dev))
        L.check_status()
        assert torch.equal(out, out2), step
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)


def test_decode_step_as_one_cuda_graph():
    # the whole step (alloc -> append -> decode) captured once and replayed: no host inputs per step
    Hq, Hkv, size, n_slots, steps = 32, 4, 8192, 16, 40
    dev = "cuda"
    kv = KvCache(size)
    perm = np.random.default_rng(9).permutation(size // 32).astype(np.uint32)
    kv.set_free_blocks(perm)
    dp = DevicePages(size, n_slots, 64, free_blocks=perm)
    kc, vc = L.alloc_cache(size, Hkv, dev), L.alloc_cache(size, Hkv, dev)
    kc2, vc2 = L.alloc_cache(size, Hkv, dev), L.alloc_cache(size, Hkv, dev)
    rope = L.rope_table(4096, dev)
    slots = torch.arange(n_slots, dtype=torch.int32, device=dev)
    q = torch.zeros(n_slots, Hq, 128, device=dev)
    k = torch.zeros(n_slots, Hkv, 128, device=dev)
    v = torch.zeros(n_slots, Hkv, 128, device=dev)
    cells = torch.empty(n_slots, dtype=torch.int64, device=dev)
    pos = torch.empty(n_slots, dtype=torch.int32, device=dev)
    ok = torch.empty(n_slots, dtype=torch.int32, device=dev)
    qr = torch.empty(n_slots, Hq, 128, device=dev)
    out = torch.empty(n_slots, Hq, 128, device=dev)
    ws = L.DecodeWorkspace(n_slots, Hq, Hkv, dev)
    def step(pages, k_cache, v_cache):
        pages.alloc_step(slots, cells, pos, ok)
        L.kv_append(k_cache, v_cache, q, k, v, pos, cells, rope, q_out=qr)
        L.attn_decode(k_cache, v_cache, qr, pages.block_tables, pages.seq_lens, out=out, workspace=ws)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up on the capture stream, on throw-away state
        step(DevicePages(size, n_slots, 64), L.alloc_cache(size, Hkv, dev), L.alloc_cache(size, Hkv, dev))
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step(dp, kc, vc)
    torch.cuda.synchronize()
    gen = torch.Generator(device=dev).manual_seed(3)
    for step in range(steps):
        q.normal_(generator=gen), k.normal_(generator=gen), v.normal_(generator=gen)
        g.replay()
        hc, hp = zip(*[kv.alloc(i, 1) for i in range(n_slots)])
        hc = torch.from_numpy(np.concatenate(hc)).to(dev)
        hp = torch.from_numpy(np.concatenate(hp)).to(dev)
        qr2 = L.kv_append(kc2, vc2, q, k, v, hp, hc, rope)
        bt, lens = kv.block_tables(np.arange(n_slots, dtype=np.int32), 64)
        out2 = L.attn_decode(kc2, vc2, qr2, torch.from_numpy(bt).to(dev), torch.from_numpy(lens).to(dev))
        L.check_status()
        assert torch.equal(cells, hc) and torch.equal(pos, hp), step
        assert torch.equal(out, out2), step
    assert int(dp.used_hwm.item()) == kv.used_hwm
    del g
