"""Evaluation harnesses (GSM8K subset scoring for the AR baseline and the block-diffusion decoder)."""
