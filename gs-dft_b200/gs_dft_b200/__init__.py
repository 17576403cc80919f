"""gs_dft_b200 — B200-native screened density-fitted Coulomb (RI-J) for Gaussian-splat DFT.

A drop-in for the RI-J hot path of andresguzco/gs-dft: the significant-pair list, the frozen
product aux with its metric and factor, the fused 3-centre fit-vector contraction, the solve and
the analytic gradient, as hand-written sm_100a CUDA kernels behind a C ABI
(``include/gsdft_b200.h``). Host code mirrors the reference's function surface.
"""
from .basis import IsotropicSplat, Splat, init_product_aux
from .coulomb import (RIJEngine, RIKEngine, aux_cholesky, aux_metric, aux_quantities,
                      df_coulomb_energy_screened, df_coulomb_gamma_screened, df_coulomb_solve,
                      df_exchange_energy_screened, screened_coulomb_energy)
from .ks import (CoulombKS, DFSpec, ExternalKS, Pairlist, ScreenedExactCoulomb, SplatModel,
                 SplatState, df, pad_rule, pairlist, refresh)
from .screening import (density_pairs, neighbor_pairs, screened_external_energy,
                        screened_nuclear_pairs, stripe_pairs)

__all__ = [
    "Splat", "IsotropicSplat", "init_product_aux", "neighbor_pairs", "stripe_pairs",
    "aux_quantities", "aux_metric", "aux_cholesky", "df_coulomb_gamma_screened",
    "df_coulomb_solve", "df_coulomb_energy_screened", "RIJEngine", "df", "pairlist", "DFSpec",
    "Pairlist", "CoulombKS", "SplatModel", "SplatState", "refresh", "pad_rule",
    "screened_nuclear_pairs", "density_pairs", "screened_external_energy", "ExternalKS",
    "RIKEngine", "df_exchange_energy_screened", "screened_coulomb_energy", "ScreenedExactCoulomb",
]
