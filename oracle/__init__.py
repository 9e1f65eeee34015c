"""CPU oracle of the FanarVSE query hot path (test infrastructure only; never imported by the product)."""
