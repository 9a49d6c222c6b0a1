"""Preprocessing helpers shared by the model pipelines (media IO)."""
