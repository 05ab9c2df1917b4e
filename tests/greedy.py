"""Greedy-token check shared by the parity tests.

The reference picks the last maximum of the logits (`Iterator::max_by` with
`total_cmp`, `engine.rs:2247-2253`). The CUDA path's logits agree with the
oracle's only within a tolerance, so when the oracle's two best logits are
closer than that tolerance either of them is a faithful greedy choice; at any
larger margin the tokens must be identical."""

import numpy as np


def reference_choice(logits) -> int:
    ref = np.asarray(logits)
    return int(np.nonzero(ref == ref.max())[0][-1])


def check_greedy(token: int, ref_logits, tol: float, where: str = "") -> bool:
    """Assert `token` is the reference's greedy choice or the other side of a
    near-tie within `tol`; returns True when it is exactly the reference's."""
    ref = np.asarray(ref_logits)
    want = reference_choice(ref)
    if int(token) == want:
        return True
    assert float(ref[int(token)]) >= float(ref.max()) - tol, \
        f"{where}: greedy token {token} (logit {ref[int(token)]}) vs reference {want} (logit {ref.max()})"
    return False
