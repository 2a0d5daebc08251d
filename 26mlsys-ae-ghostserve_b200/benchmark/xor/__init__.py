"""Drop-in replacements for the reference modules of the same path."""
