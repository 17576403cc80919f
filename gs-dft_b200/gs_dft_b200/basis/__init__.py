"""Splat bases: the full-covariance spectral chart and the isotropic density-fitting aux."""
from .spectral import Splat, full_quantities, quat_to_rotation
from .isotropic import IsotropicSplat, init_product_aux

__all__ = ["Splat", "full_quantities", "quat_to_rotation", "IsotropicSplat", "init_product_aux"]
