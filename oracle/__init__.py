"""CPU oracle of the renderer hot path (test infrastructure; see ref_restated)."""
