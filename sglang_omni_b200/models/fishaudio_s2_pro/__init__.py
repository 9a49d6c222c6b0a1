"""FishAudio S2-Pro dual-AR text-to-speech (slow AR + fast AR + DAC codec)."""
