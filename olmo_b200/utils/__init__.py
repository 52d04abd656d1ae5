"""Framework-internal helpers (typed config engine, device timing)."""
