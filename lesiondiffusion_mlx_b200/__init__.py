"""B200-native (sm_100a) hot path of lesiondiffusion-mlx: the 3-D latent
diffusion denoiser, its DDIM / DPM++-2M samplers and the VQ decoder.

Compute runs in ``libldb200.so`` (hand-written CUDA for sm_100a behind the C
ABI in ``include/ldb200.h``); PyTorch provides device memory, streams and
``torch.distributed``.  The operator names mirror the reference package's
native-kernel API so the networks read like ``lesiondiffusion_mlx``.
"""

__version__ = "0.1.0"
