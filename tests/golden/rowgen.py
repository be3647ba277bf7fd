"""Synthetic fp8 rows with a chosen exponent distribution.

Restates the row generator of the reference's tests/test_codec.py:23-46
(monochromegane/vllm-expert-pager): exponents drawn from ``p`` with
``torch.multinomial``, sign and mantissa bits uniform.
"""

import torch

EXP_P = [0.0] * 4 + [0.001, 0.002, 0.004, 0.008, 0.016, 0.032, 0.064, 0.125, 0.228, 0.315,
                     0.188, 0.015]


def rows(seed: int, n: int, p=EXP_P) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    exp = torch.multinomial(torch.tensor(p, dtype=torch.float64), n, replacement=True,
                            generator=g)
    sm = torch.randint(0, 256, (n,), dtype=torch.uint8, generator=g) & 0x87
    return sm | (exp.to(torch.uint8) << 3)
