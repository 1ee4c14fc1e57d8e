"""Op families of the B200 build: only ``sampler``."""
