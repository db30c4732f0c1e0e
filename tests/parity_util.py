"""Comparison helpers of the GPU parity tests (bf16 tolerance, posterior agreement with
near-ties logged)."""
import numpy as np
import torch


def elem_rel_err(ours: torch.Tensor, ref: torch.Tensor) -> float:
    """max over elements of |ours - ref| / max(|ref|, rms of the reference row)."""
    a = ours.float().reshape(-1, ours.shape[-1])
    b = ref.float().reshape(-1, ref.shape[-1]).to(a.device)
    rms = b.pow(2).mean(-1, keepdim=True).sqrt()
    return ((a - b).abs() / torch.maximum(b.abs(), rms).clamp_min(1e-30)).max().item()


def norm_rel_err(ours: torch.Tensor, ref: torch.Tensor) -> float:
    a, b = ours.float(), ref.float().to(ours.device)
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def posterior_agreement(label, ours, ref, ref_gap, tie_gap):
    """Fraction of decided rows (reference top-1 / top-2 gap > tie_gap, a scalar or one bound
    per row) where the posteriors agree; every disagreeing row is printed with its gap."""
    ours, ref, ref_gap = (np.asarray(x) for x in (ours, ref, ref_gap))
    tie = np.broadcast_to(np.asarray(tie_gap, dtype=np.float64), ref_gap.shape)
    decided = ref_gap > tie
    agree = ours == ref
    for i in np.flatnonzero(~agree):
        kind = "near-tie" if not decided[i] else "DECIDED"
        print(f"[{label}] row {i}: ours {ours[i]} ref {ref[i]} ref gap {ref_gap[i]:.4g} "
              f"({kind}, tie bound {tie[i]:.3g})")
    print(f"[{label}] {int(agree.sum())}/{agree.size} rows agree; {int((~decided).sum())} "
          f"near-tie rows (tie bound median {float(np.median(tie)):.3g})")
    return float(agree[decided].mean()) if decided.any() else 1.0


def walk_agrees(accepted_ref, post_ours, post_ref):
    """The walk reads the posterior only at the nodes of its path."""
    return all(int(post_ours[i]) == int(post_ref[i]) for i in accepted_ref)
