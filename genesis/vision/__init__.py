"""Vision tier (planned in the reference; no code there either)."""
