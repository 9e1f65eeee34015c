"""FanarVSE query hot path on B200 (sm_100a)."""
