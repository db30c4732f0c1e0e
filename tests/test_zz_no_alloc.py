"""The tree build entry point that allocates nothing (ddt_topk_tree_noalloc).

It exists for callers that cannot allocate device memory when they call into this
library: serving stacks that hand all device memory to their own pool at start-up and
forbid allocation afterwards, and plugin interfaces that carry only inputs and outputs,
so no workspace can be passed.  Its scratch is a fixed array in the library's device
image.  These tests call it through the C ABI and compare every output with the
workspace entry point (ddt_topk_tree) bit for bit, on two calls in a row (the second call
runs on the scratch contents the first one left behind).  The file is named so pytest
collects it last.
"""
import numpy as np
import pytest
import torch

from mdflash_b200 import _lib

pytestmark = pytest.mark.gpu

DEPTHS, VOCAB = 15, 151936


def _outputs(device, budget):
    k = min(budget, VOCAB)
    n = budget + 1
    words = (n + 31) // 32
    i64 = dict(dtype=torch.int64, device=device)
    return dict(
        top_lp=torch.full((DEPTHS, k), -1.0, dtype=torch.float32, device=device),
        top_ids=torch.full((DEPTHS, k), -1, **i64),
        node_ids=torch.full((budget,), -1, **i64),
        depths=torch.full((budget,), -1, **i64),
        parents=torch.full((n,), -7, dtype=torch.int32, device=device),
        count=torch.full((1,), -1, dtype=torch.int32, device=device),
        bits=torch.full((n, words), -1, dtype=torch.int32, device=device),
        ids=torch.full((n,), -1, **i64),
        pos=torch.full((n,), -1, **i64),
    )


def _args(logits, budget, root, out):
    return [logits.data_ptr(), _lib.DDT_BF16, DEPTHS, VOCAB, logits.stride(0), budget,
            out["top_lp"].data_ptr(), out["top_ids"].data_ptr(), out["node_ids"].data_ptr(),
            out["depths"].data_ptr(), out["parents"].data_ptr(), out["count"].data_ptr(),
            out["bits"].data_ptr(), out["bits"].shape[1], root.data_ptr(), 8192,
            out["ids"].data_ptr(), out["pos"].data_ptr()]


@pytest.mark.parametrize("budget", [256, 1024])
def test_noalloc_tree_matches_workspace_entry_point(cuda_device, budget):
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    rng = np.random.default_rng(budget)
    logits = (torch.from_numpy(rng.standard_normal((DEPTHS, VOCAB)).astype(np.float32) * 3)
              .to(torch.bfloat16).to(cuda_device))
    root = torch.tensor([77], dtype=torch.int64, device=cuda_device)

    ref = _outputs(cuda_device, budget)
    ws_bytes = lib.ddt_topk_tree_workspace_bytes(DEPTHS, VOCAB, budget)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda_device)
    rc = lib.ddt_topk_tree(*_args(logits, budget, root, ref), ws.data_ptr(), ws_bytes, stream)
    assert rc == 0, lib.ddt_error_string(rc)

    for call in range(2):
        got = _outputs(cuda_device, budget)
        rc = lib.ddt_topk_tree_noalloc(*_args(logits, budget, root, got), stream)
        assert rc == 0, lib.ddt_error_string(rc)
        torch.cuda.synchronize(cuda_device)
        for name in ref:
            assert torch.equal(got[name], ref[name]), (call, name)
        assert int(got["count"].item()) == budget


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    # 20 depths over a 262144-token vocabulary at budget 1024 needs ~2.7 MB of scratch
    assert lib.ddt_topk_tree_workspace_bytes(20, 262144, 1024) > (2 << 20)
    dummy = torch.zeros(16, dtype=torch.int64, device=cuda_device)
    p = dummy.data_ptr()
    rc = lib.ddt_topk_tree_noalloc(p, _lib.DDT_BF16, 20, 262144, 262144, 1024, p, p, p, p, p, p,
                                   p, 33, p, 0, p, p,
                                   torch.cuda.current_stream(cuda_device).cuda_stream)
    assert rc == -8
    assert b"no-alloc" in lib.ddt_error_string(rc)
