"""Drop-in for the chain sampler of the MDFlash / P-Express variants (mdflash.py of the DDTree
research code): ``sample_candidate_chains`` (mdflash.py:19-40) on the device.  Its chains
feed ``mdflash_b200.ddtree.build_sampled_candidate_tree`` (ddtree.py:169-224), whose trie
is then compiled, verified, walked and compacted by the same kernels as a best-first tree.
"""
from __future__ import annotations

import torch

from . import kernels as K


def sample_candidate_chains(draft_logits: torch.Tensor, num_samples: int,
                            proposal_temperature: float,
                            generator: torch.Generator | None = None) -> torch.Tensor:
    """mdflash.py:19-40: i64 [num_samples, depths] on the logits' device.  Chain s holds
    sample s of every depth, drawn with replacement from softmax(logits / T); below
    T = 1e-5 every chain is the argmax chain.  The draws follow torch.multinomial's
    distribution with this library's counter-based generator; its seed is taken from
    `generator` (default: torch's global CPU generator), so torch.manual_seed reproduces
    them."""
    horizon = int(draft_logits.shape[0])
    if num_samples <= 0:
        return torch.empty((0, horizon), dtype=torch.long, device=draft_logits.device)
    if horizon == 0:
        return torch.empty((num_samples, 0), dtype=torch.long, device=draft_logits.device)
    if not draft_logits.is_cuda:
        raise ValueError("draft_logits must be a CUDA tensor: mdflash_b200 runs on the GPU only")
    seed, offset = torch.randint(0, 2 ** 62, (2,), generator=generator).tolist()
    return K.sample_chains(draft_logits, num_samples, proposal_temperature, seed, offset)
