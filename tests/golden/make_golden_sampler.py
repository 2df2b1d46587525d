"""Generate the sampler golden vectors from the real reference.

    python tests/golden/make_golden_sampler.py /path/to/micro-vllm

Imports ``micro_vllm`` from ``<path>/src`` and runs, on the CPU, the
reference's own ``Sampler`` on greedy rows (src/micro_vllm/sampling/
sampler.py:14-46) and its ``_apply_top_k`` / ``_apply_top_p`` filters
(sampler.py:64-87) after the temperature division (sampler.py:48) on seeded
logits.  ``sampler_cases.npz`` holds the logits, the greedy token of every
row, and per filter case the temperature, top_k, top_p and the kept mask
(tokens the filters leave finite).  Logits are distinct within a row, so
the filters' tie order (left open by torch) does not matter; the greedy
rows include an exact tie, where torch.argmax takes the first index.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    import torch
    from micro_vllm.sampling import sampler as ref
    from micro_vllm.sampling.params import SamplingParams

    g = torch.Generator().manual_seed(5)
    rows, vocab = 6, 4096
    logits = torch.randn((rows, vocab), generator=g) * 3.0
    logits[2, 17] = logits[2, 99] = logits[2].max() + 1.0  # tie: first index wins
    greedy = ref.Sampler()(
        logits, tuple(f"r{i}" for i in range(rows)),
        tuple(SamplingParams(max_tokens=1) for _ in range(rows)), (0,) * rows,
    )
    greedy_ids = np.array([t.token_id for t in greedy.sampled_tokens], np.int64)
    cases = [(0.7, 50, 1.0), (1.0, None, 0.9), (1.3, 200, 0.5), (0.5, None, 0.05), (2.0, 1, 1.0),
             (1.0, 4096, 1.0)]
    kept = np.zeros((len(cases), rows, vocab), bool)
    for c, (temperature, top_k, top_p) in enumerate(cases):
        for r in range(rows):
            x = logits[r].to(torch.float32) / temperature
            x = ref._apply_top_k(x, top_k)
            x = ref._apply_top_p(x, top_p)
            kept[c, r] = torch.isfinite(x).numpy()
    np.savez_compressed(
        HERE / "sampler_cases.npz", logits=logits.numpy(), greedy=greedy_ids,
        temperature=np.array([c[0] for c in cases], np.float32),
        top_k=np.array([0 if c[1] is None else c[1] for c in cases], np.int32),
        top_p=np.array([c[2] for c in cases], np.float32), kept=np.packbits(kept, axis=-1),
    )
    print("wrote sampler_cases.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden_sampler.py <micro-vllm source tree>")
    main(sys.argv[1])
