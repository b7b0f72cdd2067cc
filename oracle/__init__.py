"""CPU oracle of the splat-training hot path: test infrastructure only (see oracle.py)."""
