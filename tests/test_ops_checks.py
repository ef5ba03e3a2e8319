"""Host-side size checks of the op wrappers: a buffer that a kernel indexes by
another argument's size must be large enough, or the call raises before any
launch (these run without a GPU: the size checks come before the device
checks)."""
import pytest
import torch

from heterocache_b200 import ops

i32 = torch.int32


def test_drift_check_rejects_a_short_query_buffer():
    with pytest.raises(ValueError, match="qbuf needs"):
        ops.drift_check(torch.zeros(4, 32, 128), torch.zeros(4, 256, 1, 128), torch.zeros(8, 5, dtype=i32),
                        num_kv_heads=8, groups=4, steps=5, seq_len=1000, pooling="avgpool", kernel_size=5,
                        topk=200, threshold=0.5, pivot_heads=torch.zeros(1, dtype=i32),
                        ref_slots=torch.zeros(1, dtype=i32), max_len=torch.zeros(1, dtype=i32), max_len_cap=16,
                        ref_bitmap=torch.zeros(1, 32, dtype=i32), ref_positions=torch.zeros(1, 200, dtype=i32),
                        trigger=torch.zeros(1, dtype=i32), retrieve_positions=torch.zeros(1, 16, dtype=i32),
                        workspace=None, err=torch.zeros(1, dtype=i32))


def test_drift_check_rejects_a_page_table_shorter_than_the_keys():
    with pytest.raises(ValueError, match="block_table rows"):
        ops.drift_check(torch.zeros(5, 32, 128), torch.zeros(4, 256, 1, 128), torch.zeros(8, 3, dtype=i32),
                        num_kv_heads=8, groups=4, steps=5, seq_len=1000, pooling="avgpool", kernel_size=5,
                        topk=200, threshold=0.5, pivot_heads=torch.zeros(1, dtype=i32),
                        ref_slots=torch.zeros(1, dtype=i32), max_len=torch.zeros(1, dtype=i32), max_len_cap=16,
                        ref_bitmap=torch.zeros(1, 32, dtype=i32), ref_positions=torch.zeros(1, 200, dtype=i32),
                        trigger=torch.zeros(1, dtype=i32), retrieve_positions=torch.zeros(1, 16, dtype=i32),
                        workspace=None, err=torch.zeros(1, dtype=i32))


def test_pivot_init_rejects_a_short_bitmap():
    with pytest.raises(ValueError, match="ref_bitmap needs"):
        ops.pivot_init(torch.zeros(1, 32, 1, 128), torch.zeros(1, 8, 3000, 128), first_pivot=7, n_pivots=1,
                       groups=4, pooling="avgpool", kernel_size=5, topk=600,
                       ref_positions=torch.zeros(1, 1, 600, dtype=i32), ref_bitmap=torch.zeros(1, 1, 93, dtype=i32),
                       workspace=None, err=torch.zeros(1, dtype=i32))


def test_prefill_select_rejects_short_outputs():
    with pytest.raises(ValueError, match="out_indices needs"):
        ops.prefill_select(torch.zeros(1, 32, 1, 128), torch.zeros(1, 8, 1000, 128), torch.zeros(1, 8, 1000, 128),
                           torch.zeros(3, dtype=i32), 400, n_heads=3, groups=4, window=1, pooling="avgpool",
                           kernel_size=5, k_pool=torch.zeros(4, 256, 1, 128), v_pool=torch.zeros(4, 256, 1, 128),
                           block_table=torch.zeros(8, 5, dtype=i32), heads_len=torch.zeros(8, dtype=i32),
                           workspace=None, err=torch.zeros(1, dtype=i32), out_indices=torch.zeros(1, 3, 399, dtype=i32))


def test_retrieve_rejects_position_rows_shorter_than_the_members():
    with pytest.raises(ValueError, match="retrieve_positions rows"):
        ops.retrieve(member_job=torch.zeros(2, dtype=i32), member_head=torch.zeros(2, dtype=i32),
                     member_len=torch.zeros(2, dtype=i32), max_member_len=400, trigger=torch.zeros(1, dtype=i32),
                     retrieve_positions=torch.zeros(1, 300, dtype=i32), full_k=torch.zeros(1, 8, 1000, 128),
                     full_v=torch.zeros(1, 8, 1000, 128), k_pool=torch.zeros(4, 256, 1, 128),
                     v_pool=torch.zeros(4, 256, 1, 128), block_table=torch.zeros(8, 5, dtype=i32), num_kv_heads=8,
                     err=torch.zeros(1, dtype=i32))


def test_flash_decode_rejects_query_heads_that_do_not_split_over_the_kv_heads():
    """30 query heads over 8 KV heads: the kernels would write only 8 x 3 of
    the 30 output heads, so the call raises before allocating or launching."""
    with pytest.raises(ValueError, match="do not split evenly"):
        ops.flash_decode(torch.zeros(1, 30, 1, 128), torch.zeros(4, 256, 1, 128), torch.zeros(4, 256, 1, 128),
                         torch.zeros(8, 5, dtype=i32), torch.zeros(8, dtype=i32), num_kv_heads=8, workspace=None,
                         err=torch.zeros(1, dtype=i32))


def test_batch_view_of_rows_of_one_buffer():
    """attention_together's batching of the members' pending k/v and queries:
    rows of one buffer give a strided view over all of them (no copy);
    tensors of their own give None (the caller concatenates)."""
    from heterocache_b200.cache import _batch_view
    buf = torch.arange(4 * 3 * 8 * 2, dtype=torch.float32).reshape(4, 1, 3, 8, 2)
    rows = [buf[i] for i in range(4)]
    v = _batch_view(rows)
    assert v is not None and v.shape == (4, 3, 8, 2) and torch.equal(v, buf[:, 0])
    sub = [buf[i, :, 1:] for i in range(4)]  # strided rows: still one view
    assert torch.equal(_batch_view(sub), buf[:, 0, 1:])
    assert _batch_view([r.clone() for r in rows]) is None
    assert _batch_view([rows[0], rows[2], rows[1]]) is None
    assert _batch_view(rows[:1]) is rows[0]


def test_peer_put_rejects_too_many_segments_or_destinations():
    seg = torch.zeros(4, dtype=i32)
    with pytest.raises(ValueError, match="1 to 4 segments"):
        ops.peer_put([seg] * 5, [0])
    with pytest.raises(ValueError, match="at most 8 destinations"):
        ops.peer_put([seg], [16] * 9)


def test_cache_group_storage_gives_each_member_its_own_id_range():
    """CacheGroup's host side (no kernel runs): one pool per layer sized for
    every member, each member's page ids an offset range of its own, its
    page table and lengths rows of shared tensors; members needing more
    pages than the first one, or adopted after their prefill, are refused."""
    import types
    from heterocache_b200.cache import CacheGroup
    members = [types.SimpleNamespace(key_pools=[None], head_dim=128) for _ in range(3)]
    g = CacheGroup(members)
    assert [m._gidx for m in members] == [0, 1, 2] and all(m._group is g for m in members)
    out = [g._layer_storage(m, 0, 10, 8, 6, "cpu", torch.bfloat16) for m in members]
    kp0, vp0 = out[0][0], out[0][1]
    assert kp0.shape == (30, 256, 1, 128) and vp0.shape == kp0.shape
    assert [o[2] for o in out] == [0, 10, 20]
    for i, (kp, vp, off, bt, hl) in enumerate(out):
        assert kp is kp0 and vp is vp0
        assert bt.shape == (8, 6) and hl.shape == (8,)
        bt.fill_(i)
        hl.fill_(i + 1)
    st = g._layers[0]
    assert st["bt"][8:16].unique().tolist() == [1] and st["hl"][16:].unique().tolist() == [3]
    with pytest.raises(ValueError, match="different pages"):
        g._layer_storage(members[1], 0, 11, 8, 6, "cpu", torch.bfloat16)
    with pytest.raises(ValueError, match="different pages"):
        g._layer_storage(members[1], 0, 10, 8, 7, "cpu", torch.bfloat16)
    q = [g._query_buffer(m, 0, 5, 32, 128, torch.bfloat16, "cpu") for m in members]
    assert q[2].data_ptr() == g._qbufs[0][2].data_ptr() and q[0].shape == (5, 32, 128)
    late = types.SimpleNamespace(key_pools=[torch.zeros(1)], head_dim=128)
    with pytest.raises(RuntimeError, match="before their prefill"):
        CacheGroup([late])
