"""Model families built on the sm_100a kernels (random-init capable, offload-ready)."""
