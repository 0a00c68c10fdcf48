"""Layer drivers at the backends' hook points (GPTQModel, QUIP#)."""
