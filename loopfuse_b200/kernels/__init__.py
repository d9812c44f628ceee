"""Names the reference's kernel-selection table points at, resolved to sm_100a code."""
