"""Internals of the B200 BoaConstrictor hot path (native bindings, container,
weights, synthetic inputs).  The drop-in modules one directory up (``boa``,
``codec``, ``model``, ``gpu_range_coder``) are the public surface."""
