"""Model families built on the sm_100a kernels (random-init capable, offload-ready):
Wan2.2-14B-shape and LTX-shape video DiTs (``wan``, ``ltx``), a Llama-3-shape decoder
(``llama``) and a Mixtral-shape sparse-MoE decoder (``mixtral``)."""
