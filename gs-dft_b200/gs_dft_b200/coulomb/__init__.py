"""Density-fitted Coulomb (RI-J) and exchange (RI-K) on the frozen product aux: metric, factor,
fused gamma, solve and the analytic reverse passes, all on the GPU."""
from .engine import RIJEngine, make_plan, splat_quantities, check_device_status
from .exchange import RIKEngine, df_exchange_energy_screened
from .stream import screened_coulomb_energy
from .ri import (aux_cholesky, aux_metric, aux_quantities, df_coulomb_energy_screened,
                 df_coulomb_gamma_screened, df_coulomb_solve, shift_diag)

__all__ = ["RIJEngine", "make_plan", "splat_quantities", "check_device_status", "aux_cholesky",
           "aux_metric", "aux_quantities", "df_coulomb_energy_screened",
           "df_coulomb_gamma_screened", "df_coulomb_solve", "shift_diag", "RIKEngine",
           "df_exchange_energy_screened", "screened_coulomb_energy"]
