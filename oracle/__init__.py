"""CPU oracle of the block-FP8 linear path. Test infrastructure only (see oracle.oracle)."""
