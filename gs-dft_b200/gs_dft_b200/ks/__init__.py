"""Strategy specs, refresh state and the Coulomb builder (the drop-in surface of gs_dft.ks)."""
from .terms import (DFSpec, Pairlist, SCREEN_PAD, ScreenedExactCoulomb, ScreenedProductDFCoulomb,
                    df, pairlist)
from .state import CoulombKS, ExternalKS, SplatModel, SplatState, pad_rule, refresh

__all__ = ["DFSpec", "Pairlist", "SCREEN_PAD", "ScreenedProductDFCoulomb", "ScreenedExactCoulomb",
           "df", "pairlist",
           "CoulombKS", "ExternalKS", "SplatModel", "SplatState", "pad_rule", "refresh"]
