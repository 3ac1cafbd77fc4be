"""CPU oracle of the hexkernels hot path -- test infrastructure only."""
