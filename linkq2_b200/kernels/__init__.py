"""GPU operators with the signatures of the reference's ``qslab.kernels``."""
