"""Device ops: the sm_100a transfer kernels and their host-side launchers."""
