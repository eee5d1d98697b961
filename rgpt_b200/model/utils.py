"""Initialisation helpers (model/utils.py:5-37 of the reference)."""
import math

import torch


def trunc_normal_init_(tensor: torch.Tensor, std: float = 1.0, lower: float = -2.0, upper: float = 2.0):
    """Truncated normal with the variance correction that makes the result's std equal `std`.

    Same sampling procedure as the reference (inverse-CDF: uniform in [erf(l/sqrt2), erf(u/sqrt2)],
    erfinv, scale, clip), so a seeded init reproduces the reference's values (model/utils.py:5-37)."""
    with torch.no_grad():
        if std == 0:
            return tensor.zero_()
        r2 = math.sqrt(2.0)
        lo_cdf, hi_cdf = math.erf(lower / r2), math.erf(upper / r2)
        z = (hi_cdf - lo_cdf) / 2
        c = 1.0 / math.sqrt(2 * math.pi)
        pdf_lo_side = c * math.exp(-0.5 * lower ** 2)
        pdf_hi_side = c * math.exp(-0.5 * upper ** 2)
        var = 1 - (upper * pdf_lo_side - lower * pdf_hi_side) / z - ((pdf_lo_side - pdf_hi_side) / z) ** 2
        comp_std = std / math.sqrt(var)
        tensor.uniform_(lo_cdf, hi_cdf)
        tensor.erfinv_()
        tensor.mul_(r2 * comp_std)
        tensor.clip_(lower * comp_std, upper * comp_std)
    return tensor
