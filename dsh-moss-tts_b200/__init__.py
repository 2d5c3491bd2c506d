"""moss_b200 -- B200-native engine for MOSS-TTS-Nano's per-frame LLM step (placeholder)."""
