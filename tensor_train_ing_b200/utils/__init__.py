"""Small shared helpers (timing, hashing, file publishing)."""
