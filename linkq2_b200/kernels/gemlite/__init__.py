"""W4A16 linear: same module path and call signatures as the reference's
``qslab.kernels.gemlite`` (``ops.linear``, ``bitpack.pack_weights_over_cols``)."""
