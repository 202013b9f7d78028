from .rewards import latent_mlp_score, multi_score, videoalign_score  # noqa: F401
