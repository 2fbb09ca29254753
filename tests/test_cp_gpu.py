"""Context-parallel attention kernels, emulated on one GPU (GPU).

Two cache tensors stand in for two ranks' page shards: logical page i of a
sequence lives on rank i % C at physical page i // C (a CP block = C pages,
one per rank). Prefill: each rank's query tokens are the ones on its pages;
the kernel reads every page from its owner's cache. Decode: each rank attends
over its own pages, the split partials of all ranks are merged.
"""
import pytest
import torch

from k8v4_xpu_b200 import ops
from k8v4_xpu_b200.kv import oracle as O
from k8v4_xpu_b200.kv.layout import b200_layout
from k8v4_xpu_b200.kv.pack import store_tokens

pytestmark = pytest.mark.gpu


def _sharded(n, C, hkv=4, gqa=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    lay = b200_layout(hkv, gqa)
    npg = (n + 15) // 16
    per_rank = (npg + C - 1) // C + 2
    caches = [torch.zeros(per_rank, lay.page_bytes, dtype=torch.uint8) for _ in range(C)]
    k = torch.randn(n, hkv, 128, generator=g).bfloat16()
    v = torch.randn(n, hkv, 128, generator=g).bfloat16()
    for r in range(C):
        toks = [t for t in range(n) if (t // 16) % C == r]
        if toks:
            slots = torch.tensor([((t // 16) // C) * 16 + t % 16 for t in toks])
            store_tokens(caches[r], slots, k[toks], v[toks], lay)
    table = torch.tensor([((i % C) << 24) | (i // C) for i in range(npg)], dtype=torch.int32)
    kd, vd = O.quant_dequant_kv(k, v, lay)
    return lay, [c.cuda() for c in caches], table, kd, vd


@pytest.mark.parametrize("C", [2, 4])
def test_cp_prefill_reads_every_owner(C):
    n, q_len = 2000, 700          # the chunk: the sequence's last 700 tokens
    lay, caches, table, kd, vd = _sharded(n, C)
    g = torch.Generator().manual_seed(9)
    q = torch.randn(q_len, lay.hkv * lay.gqa, 128, generator=g).bfloat16()
    base = n - q_len
    ref = O.attention_ref(q.float(), kd, vd, [base + t + 1 for t in range(q_len)], lay.gqa)
    for r in range(C):
        mine = [t for t in range(q_len) if ((base + t) // 16) % C == r]
        qr = q[mine].cuda()
        pos = torch.tensor([base + t for t in mine], dtype=torch.int32, device="cuda")
        out = ops.prefill_attn_cp(qr, torch.tensor([0, len(mine)], dtype=torch.int32, device="cuda"),
                                  torch.tensor([n], dtype=torch.int32, device="cuda"), table.view(1, -1).cuda(),
                                  caches, lay.hkv, lay.gqa, len(mine), q_pos=pos)
        torch.cuda.synchronize()
        err = (out.float().cpu() - ref[mine]).abs().max().item()
        assert err < 3e-2, (r, err)
    assert ops.status() == 0


@pytest.mark.parametrize("C", [2, 4])
def test_cp_decode_partials_merge_across_ranks(C):
    n = 3001
    lay, caches, table, kd, vd = _sharded(n, C, seed=3)
    g = torch.Generator().manual_seed(4)
    q = torch.randn(1, lay.hkv * lay.gqa, 128, generator=g).bfloat16().cuda()
    cu = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    npg = (n + 15) // 16
    nsplit = 3
    rank_floats = ops.decode_ws_floats(1, lay.hkv, nsplit, 1, lay.gqa)
    ws_all = torch.empty(C * rank_floats, dtype=torch.float32, device="cuda")
    for r in range(C):
        local = [i // C for i in range(npg) if i % C == r]                  # this rank's pages, in order
        keys = sum(min(16, n - i * 16) for i in range(npg) if i % C == r)   # only the last page is partial
        out = torch.empty_like(q)
        ops.decode_attn(q, cu, torch.tensor([keys], dtype=torch.int32, device="cuda"),
                        torch.tensor(local, dtype=torch.int32, device="cuda").view(1, -1), caches[r], lay.hkv,
                        lay.gqa, 1, nsplit=nsplit, out=out, ws=ws_all[r * rank_floats:(r + 1) * rank_floats])
    merged = torch.empty_like(q)
    ops.decode_combine_ranks(ws_all, rank_floats, cu, C, nsplit, lay.hkv, lay.gqa, 1, merged)
    torch.cuda.synchronize()
    ref = O.attention_ref(q.float().cpu(), kd, vd, [n], lay.gqa)
    err = (merged.float().cpu() - ref).abs().max().item()
    assert err < 2e-2, err
    assert ops.status() == 0


def test_cp_push_exchange_one_rank_matches_the_workspace_path():
    """The partial exchange fused into the decode kernel (multicast stores,
    one signal per CTA, merge behind a bounded wait), on a one-rank group:
    the merge's wait is met by the attention kernel before it in the stream.
    Its output equals the workspace path's bit for bit, and the running
    counts advance by one call's signals per use of each buffer."""
    import socket
    import torch.distributed as dist
    from k8v4_xpu_b200.parallel.cp_combine import PeerCombine, max_slot_floats
    n = 3001
    lay, caches, table, kd, vd = _sharded(n, 1, seed=5)
    g = torch.Generator().manual_seed(6)
    q = torch.randn(2, lay.hkv * lay.gqa, 128, generator=g).bfloat16().cuda()
    cu = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    lens = torch.tensor([n, n - 700], dtype=torch.int32, device="cuda")
    bt = table.cuda().view(1, -1).repeat(2, 1).contiguous()
    nsplit = 5
    ref = ops.decode_attn(q, cu, lens, bt, caches[0], lay.hkv, lay.gqa, 1, nsplit=nsplit)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    own_group = not dist.is_initialized()
    if own_group:
        dist.init_process_group("nccl", init_method="tcp://127.0.0.1:%d" % port, rank=0, world_size=1,
                                device_id=torch.device("cuda", 0))
    try:
        try:
            peer = PeerCombine(dist.group.WORLD, torch.device("cuda", 0), max_slot_floats(2, lay.hkv, 1, lay.gqa))
        except (RuntimeError, ValueError, NotImplementedError) as e:  # no one-rank multicast object here
            pytest.skip("symmetric-memory multicast at one rank: %s" % e)
        expected = ops.decode_push_ctas(2, lay.hkv, nsplit)
        for call in range(3):  # buffers 0, 1, 0
            out = peer.attention(q, cu, lens, bt, caches[0], lay.hkv, lay.gqa, 1, nsplit)
            torch.cuda.synchronize()
            assert ops.status() == 0
            assert torch.equal(out, ref), call
        assert peer.state[:, 0].tolist() == [2 * expected, expected]
        assert peer.state[:, 1].tolist() == [0, 0]
        del peer
    finally:
        if own_group:
            dist.destroy_process_group()


@pytest.mark.parametrize("C", [2, 4])
def test_cp_verify_rows_with_local_visible_ends_merge_across_ranks(C):
    """MTP verify under context parallelism: 7 query rows of one sequence at
    its last 7 positions; on each rank row p sees the rank's first
    ``local_keys(p + 1)`` local keys (the kernel's per-row ``q_ends``), and
    the ranks' split partials merge into causal attention over every key."""
    from k8v4_xpu_b200.parallel.cp import local_keys
    n, w = 3001, 7
    lay, caches, table, kd, vd = _sharded(n, C, seed=11)
    g = torch.Generator().manual_seed(12)
    q = torch.randn(w, lay.hkv * lay.gqa, 128, generator=g).bfloat16().cuda()
    cu = torch.tensor([0, w], dtype=torch.int32, device="cuda")
    npg = (n + 15) // 16
    nsplit = 3
    pos = list(range(n - w, n))
    rank_floats = ops.decode_ws_floats(1, lay.hkv, nsplit, w, lay.gqa)
    ws_all = torch.empty(C * rank_floats, dtype=torch.float32, device="cuda")
    for r in range(C):
        local = [i // C for i in range(npg) if i % C == r]
        ends = torch.tensor([local_keys(p + 1, r, C) for p in pos], dtype=torch.int32, device="cuda")
        out = torch.empty_like(q)
        ops.decode_attn(q, cu, torch.tensor([local_keys(n, r, C)], dtype=torch.int32, device="cuda"),
                        torch.tensor(local, dtype=torch.int32, device="cuda").view(1, -1), caches[r], lay.hkv,
                        lay.gqa, w, nsplit=nsplit, out=out, ws=ws_all[r * rank_floats:(r + 1) * rank_floats],
                        q_ends=ends)
    merged = torch.empty_like(q)
    ops.decode_combine_ranks(ws_all, rank_floats, cu, C, nsplit, lay.hkv, lay.gqa, w, merged)
    torch.cuda.synchronize()
    ref = O.attention_ref(q.float().cpu(), kd, vd, [p + 1 for p in pos], lay.gqa)
    err = (merged.float().cpu() - ref).abs().max().item()
    assert err < 2e-2, err
    assert ops.status() == 0
