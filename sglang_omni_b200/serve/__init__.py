from .launcher import build_server, launch_server
from .openai_api import create_app

__all__ = ["build_server", "launch_server", "create_app"]
