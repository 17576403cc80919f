"""Significant-overlap pair screening and the screened nuclear attraction on the device."""
from .nuclear import (atom_records, density_pairs, screened_external_energy,
                      screened_nuclear_pairs)
from .pairs import count_significant, neighbor_pairs, pair_weight, stripe_pairs

__all__ = ["neighbor_pairs", "count_significant", "pair_weight", "stripe_pairs",
           "screened_nuclear_pairs", "density_pairs", "screened_external_energy", "atom_records"]
