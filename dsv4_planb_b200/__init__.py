"""B200-native ``sparse_attn_sharedkv`` (DeepSeek-V4 style shared K=V latent attention)."""
