"""The decode loop on the GPU path against the reference's own loop.

``tests/golden/make_golden.py`` ran the reference's ddtree_generate (ddtree.py:338-530) on the
CPU, fp32, with a tiny Qwen3 target and a deterministic stand-in for the drafter, for 20 rounds
that each accept two tokens.  ``mdflash_b200.generate.ddtree_generate`` runs the same loop on
the GPU through this package's tree build, compile, attention plug-in, argmax, walk and
compaction (attention in bf16 inside the fp32 model).  The committed tokens and the per-round
acceptance lengths must be identical.
"""
import numpy as np
import pytest
import torch

import inputs as gin
from mdflash_b200.generate import ddtree_generate

pytestmark = pytest.mark.gpu


def test_decode_loop_matches_reference_loop(golden, cuda_device):
    spec = gin.LOOP_CASE
    target = gin.loop_target(spec).to(cuda_device)
    drafter = gin.StubDrafter(spec["hidden"]).to(cuda_device)
    ids = gin.loop_inputs(spec).to(cuda_device)
    res = ddtree_generate(drafter, target, ids, spec["mask_token_id"], spec["max_new_tokens"],
                          spec["block_size"], None, 0.0, spec["budget"])
    torch.cuda.synchronize()
    print(f"[loop] acceptance {res.acceptance_lengths}")
    assert res.acceptance_lengths == golden["loop/acceptance_lengths"].tolist()
    np.testing.assert_array_equal(res.output_ids.numpy(), golden["loop/output_ids"])
    assert res.num_output_tokens == golden["loop/output_ids"].shape[1] - spec["prompt"]
