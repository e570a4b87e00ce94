"""Drop-in for the reference's native module package (``lema._csrc``)."""
