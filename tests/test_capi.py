"""CPU checks of the C-ABI boundary: the library loads and exports every entry point
declared in include/ddtree_b200.h with the binding's signature; argument validation
that happens on the host returns the documented error codes without touching a GPU."""
import ctypes
import os
import re

import pytest

from mdflash_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "ddtree_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ddt_[a-z0-9_]+)\s*\(", src)))


def test_header_and_binding_agree():
    assert _declared() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name


def test_error_strings_and_version():
    lib = _lib.load()
    assert lib.ddt_version() >= 1
    for code in (0, -1, -2, -3, -4, -5, -6, -7, -8):
        assert lib.ddt_error_string(code)
    assert lib.ddt_error_string(-99) == b"unknown error"


def test_host_side_validation_rejects_bad_arguments():
    lib = _lib.load()
    # capacity: budget above the compiled limit, before any device work
    rc = lib.ddt_topk_tree(None, 1, 15, 1000, 1000, 5000, None, None, None, None,
                           ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 200,
                           None, 0, None, None, None, 0, None)
    assert rc == -2
    rc = lib.ddt_topk_tree(None, 7, 15, 1000, 1000, 8, None, None, None, None,
                           ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 1,
                           None, 0, None, None, None, 0, None)
    assert rc == -3
    # attention: head_dim other than 128 is a capacity error, odd GQA ratio invalid
    assert lib.ddt_tree_attn(ctypes.c_void_p(256), 128, 128, ctypes.c_void_p(256),
                             ctypes.c_void_p(256), 128, 128, ctypes.c_void_p(256), 128, 128, 4,
                             0, 4, 2, 64, ctypes.c_void_p(256), 1, 0, 1.0, 0, None, 0, None,
                             None) == -2
    assert lib.ddt_tree_attn(ctypes.c_void_p(256), 128, 128, ctypes.c_void_p(256),
                             ctypes.c_void_p(256), 128, 128, ctypes.c_void_p(256), 128, 128, 4,
                             0, 6, 4, 128, ctypes.c_void_p(256), 1, 0, 1.0, 0, None, 0, None,
                             None) == -1
    # compaction: more kept rows than a tree can accept
    assert lib.ddt_compact_kv(ctypes.c_void_p(256), 64, ctypes.c_void_p(256), 2, 2, 128, 1024,
                              128, 2, 10, None) == -2
    assert lib.ddt_argmax(None, 2, 4, 4, 4, None, None) == -3
    # sampled-chain trie: more chains than a tree budget holds is a capacity error
    assert lib.ddt_chain_tree(p := ctypes.c_void_p(256), 2000, 15, 15, 64, p, p, p, p, p, 3,
                              None, 0, None, None, None) == -2
    assert lib.ddt_sample_chains(ctypes.c_void_p(256), 1, 21, 100, 100, 8, 1.0, 0, 0,
                                 ctypes.c_void_p(256), None) == -2
    assert lib.ddt_sample_chains(ctypes.c_void_p(256), 5, 4, 100, 100, 8, 1.0, 0, 0,
                                 ctypes.c_void_p(256), None) == -3
    # fused lm_head -> argmax: hidden size a multiple of 64, a large enough workspace
    assert lib.ddt_lm_head_argmax(p, 100, p, 100, 8, 100, 1000, p, None, 0, p, 4096, None,
                                  None) == -2
    assert lib.ddt_lm_head_argmax(p, 128, p, 128, 8, 128, 1000, p, None, 0, p, 16, None,
                                  None) == -7
    assert lib.ddt_lm_head_argmax_workspace_bytes(257) >= 257 * 8 + 4
    # batched tree build: budget / depth limits, per-request budgets required, a workspace of
    # one slice per request
    bt = lib.ddt_topk_tree_batched
    assert bt(p, 1, 4, 15, 1000, 1000, 15000, p, 2000, p, p, p, p, p, 63, None, None, None,
              None, p, 1 << 30, None) == -2
    assert bt(p, 1, 4, 15, 1000, 1000, 15000, None, 64, p, p, p, p, p, 3, None, None, None,
              None, p, 1 << 30, None) == -1
    assert bt(p, 1, 4, 15, 1000, 1000, 100, p, 64, p, p, p, p, p, 3, None, None, None,
              None, p, 1 << 30, None) == -1  # requests overlap
    ws1 = lib.ddt_topk_tree_batched_workspace_bytes(1, 15, 1000, 64)
    ws4 = lib.ddt_topk_tree_batched_workspace_bytes(4, 15, 1000, 64)
    slice_ = lib.ddt_topk_tree_workspace_bytes(15, 1000, 64)
    assert ws1 >= slice_ and 4 * slice_ <= ws4 < 4 * ws1
    assert bt(p, 1, 4, 15, 1000, 1000, 15000, p, 64, p, p, p, p, p, 3, None, None, None,
              None, p, ws4 - 1, None) == -7
    assert bt(p, 1, 0, 15, 1000, 1000, 15000, p, 64, p, p, p, p, p, 3, None, None, None,
              None, p, 0, None) == 0
    # fused elementwise stages: head_dim 128 only, a 16-byte aligned rope table, hidden up to
    # 16384 in multiples of 8
    assert lib.ddt_rope_table(p, 4, p, 64, 1.0, p, None) == -2
    assert lib.ddt_rope_table(p, 4, p, 128, 1.0, ctypes.c_void_p(260), None) == -4
    assert lib.ddt_rope_table(None, 4, p, 128, 1.0, p, None) == -1
    assert lib.ddt_qk_norm_rope_cache_table(p, 4, 32, 8, 128, p, p, 1e-6, None, p, p, p, 1024,
                                            128, 0, None) == -1
    assert lib.ddt_qk_norm_rope_cache_table(p, 4, 32, 8, 128, p, p, 1e-6, ctypes.c_void_p(264),
                                            p, p, p, 1024, 128, 0, None) == -4
    assert lib.ddt_add_rmsnorm(p, None, p, 4, 16392, 1e-6, None, p, None) == -2
    assert lib.ddt_add_rmsnorm(p, None, p, 4, 100, 1e-6, None, p, None) == -2
    assert lib.ddt_add_rmsnorm(p, None, p, 0, 5120, 1e-6, None, p, None) == 0
    # NVLink peer exchange: at most 8 ranks, head_dim 128, epochs from 1, bounded waits
    assert lib.ddt_peer_buffer_bytes(9, 513, 32, 128) == 0
    assert lib.ddt_peer_buffer_bytes(2, 513, 32, 64) == 0
    assert lib.ddt_peer_buffer_bytes(2, 513, 32, 128) > 2 * 2 * 513 * 32 * 130 * 4
    bases = (ctypes.c_void_p * 2)(256, 512)
    pb = ctypes.cast(bases, ctypes.c_void_p)
    assert lib.ddt_peer_push(p, p, p, 513, 32, 128, pb, 9, 0, 1, p, None) == -2
    assert lib.ddt_peer_push(p, p, p, 513, 32, 128, pb, 2, 2, 1, p, None) == -1
    assert lib.ddt_peer_push(p, p, p, 513, 32, 128, pb, 2, 0, 0, p, None) == -1
    assert lib.ddt_peer_merge(p, 2, 513, 32, 128, 1, p, 4096, 128, p, 10, None) == -1
    assert lib.ddt_peer_merge(p, 2, 513, 32, 128, 1, p, 4096, 128, None, 10**6, None) == -1
    assert lib.ddt_peer_alloc(0, None, None) == -1
    # the bounded-wait check takes limits from 100 us to 2 s and needs a status word
    p = ctypes.c_void_p(256)
    assert lib.ddt_tree_attn_wait_check(p, p, p, p, 65, 256, 32, 8, p, 3, 10, p, None) == -1
    assert lib.ddt_tree_attn_wait_check(p, p, p, p, 65, 256, 32, 8, p, 3, 10**6, None, None) == -1


def test_workspace_queries():
    lib = _lib.load()
    ws = lib.ddt_topk_tree_workspace_bytes(15, 151936, 256)
    chunks = -(-151936 // 20480)  # 20480-element chunks per depth row
    assert ws > 15 * chunks * 256 * 8  # candidates of every chunk
    assert lib.ddt_tree_attn_workspace_bytes(257, 32, 128, 2) >= 2 * 257 * 32 * 130 * 4


@pytest.mark.parametrize("n,past,expect", [
    # 256 query rows (64 nodes x 4 grouped heads) per CTA: 8 heads x 5 row pairs = 40 CTAs
    # per split, 148 // 40 = 3 splits of the 66 key tiles
    (257, 8192, 3),
    # 8 x 9 = 72 CTAs per split -> 2 splits
    (513, 131072, 2),
    # key range too short for more than one split of >= 4 tiles
    (65, 300, 1)])
def test_attention_split_count(n, past, expect):
    from mdflash_b200.kernels import attn_splits
    assert attn_splits(n, 32, 8, past) == expect
    assert attn_splits(n, 32, 8, past, kv_splits=5) == 5


def _plan(n, past, hq, hkv, splits=0, key_begin=0, key_end=-1):
    import ctypes
    from mdflash_b200 import _lib
    out = (ctypes.c_int64 * 4)()
    rc = _lib.load().ddt_tree_attn_plan(n, past, hq, hkv, splits, key_begin, key_end,
                                        ctypes.cast(out, ctypes.c_void_p))
    return rc, list(out)


def test_attention_plan_known_shapes():
    # Qwen3-8B verify shape: 40 units of 256 rows, balanced over all 148 SMs, merged
    rc, plan = _plan(257, 8192, 32, 8)
    assert rc == 0 and plan[0] == 1 and plan[1] == 148 and plan[2] >= 148
    # 131072-key prefix: K / V beyond L2, uniform key splits
    rc, plan = _plan(513, 131072, 32, 8)
    assert rc == 0 and plan[0] == 0 and plan[2] > 1 and plan[1] <= 148
    # explicit splits stay uniform
    rc, plan = _plan(257, 8192, 32, 8, 3)
    assert rc == 0 and plan == [0, 40 * 3, 3, 1]
    # sizes the kernel rejects
    assert _plan(0, 8192, 32, 8)[0] == -1
    assert _plan(257, 8192, 32, 7)[0] == -1


def test_attention_balanced_tables_cover_every_tile():
    """The balanced scheduler (fitted cost model) checks its own table: each key tile of each
    work unit in exactly one item, a unit's items in key order.  Swept over tree sizes,
    prefix lengths (tile multiples and not) and head layouts."""
    seen_balanced = 0
    for hq, hkv in [(32, 8), (16, 8), (8, 8), (4, 1), (8, 2)]:
        for n in [1, 2, 17, 33, 64, 65, 100, 129, 257, 300, 513, 1025]:
            for past in [0, 1, 37, 127, 128, 1000, 4096, 8192, 16384, 32768, 65536, 131072]:
                rc, plan = _plan(n, past, hq, hkv)
                assert rc == 0, (hq, hkv, n, past, rc)
                assert 1 <= plan[1] <= (148 if plan[0] else 1 << 20)
                if plan[0]:
                    seen_balanced += 1
                    assert plan[2] >= 1 and plan[3] >= 1
    assert seen_balanced > 100


def test_attention_shard_tables_cover_every_tile():
    """The same check for the key shards of a split-KV call (ddt_tree_attn_partial_merged):
    2, 4 and 8 contiguous shards of the prefix, the last one holding the tree keys."""
    seen_balanced = 0
    for hq, hkv in [(32, 8), (16, 8)]:
        for n in [17, 65, 257, 513]:
            for past in [1000, 8192, 32768, 131072]:
                total = past + n
                for world in (2, 4, 8):
                    step = past // world
                    for r in range(world):
                        b = r * step
                        e = total if r == world - 1 else (r + 1) * step
                        rc, plan = _plan(n, past, hq, hkv, 0, b, e)
                        assert rc == 0, (hq, hkv, n, past, world, r, rc)
                        seen_balanced += plan[0]
    assert seen_balanced > 50
    # a shard outside the key range is rejected
    assert _plan(65, 1000, 32, 8, 0, 500, 2000)[0] == -1


def test_attention_shard_plans_report_their_merge():
    """A shard's result is always one merged partial per row, so a shard plan reports at
    least one part to merge, and an empty shard is planned as a shard, not as the full range."""
    # the first shard of a prefix beyond L2 with few key tiles per unit: uniform splits
    for b, e in [(0, 512), (0, 131072 // 8), (0, 128)]:
        rc, plan = _plan(513, 131072, 32, 8, 0, b, e)
        assert rc == 0 and plan[2] >= 1, (b, e, plan)
    rc, plan = _plan(257, 300000, 32, 8, 0, 0, 300000)
    assert rc == 0 and plan[0] == 0 and plan[2] >= 1
    # the empty shard [0, 0) (rank 0's shard of an empty prefix): uniform, one part, merged
    rc, plan = _plan(65, 0, 32, 8, 0, 0, 0)
    assert rc == 0 and plan == [0, 8 * 2, 1, 1]
    # the full-range call of the same sizes: one launch, nothing to merge
    rc, plan = _plan(65, 0, 32, 8)
    assert rc == 0 and plan[2] == 0


@pytest.mark.parametrize("depths,vocab,budget,expect", [
    (15, 151936, 256, 256), (3, 3, 40, 39), (0, 10, 5, 0), (15, 10, 0, 0), (1, 1000, 8, 8),
    (2, 4, 100, 20)])
def test_expected_node_count(depths, vocab, budget, expect):
    from mdflash_b200.kernels import expected_node_count
    assert expected_node_count(depths, vocab, budget) == expect
