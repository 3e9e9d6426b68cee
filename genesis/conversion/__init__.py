"""Model conversion (planned in the reference; no code there either)."""
