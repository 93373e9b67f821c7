"""``jax.experimental`` stand-in: Pallas is imported by the reference's kernel module but never run here."""
