"""CPU oracle of the parakeet.wgsl encoder hot path (test infrastructure only)."""
