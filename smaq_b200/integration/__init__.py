"""Framework integrations (smaq/integration in the reference)."""
