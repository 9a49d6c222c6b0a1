"""``sgl-omni-b200`` command line: ``serve`` and ``config view|export``
(same verbs and flags as sglang_omni/cli/cli.py:6-12, serve.py:15-83,
config.py:19-76)."""
from __future__ import annotations

import argparse
import logging
import sys

from ..config import ConfigManager


def _load(args, extra):
    if args.config:
        cfg = ConfigManager.from_file(args.config)
    else:
        if not args.model_path:
            raise SystemExit("--model-path or --config is required")
        cfg = ConfigManager.from_model_path(args.model_path, variant="text" if getattr(args, "text_only", False)
                                            else None)
    overrides = ConfigManager.parse_extra_args(extra)
    if overrides:
        cfg = ConfigManager.merge_config(cfg, overrides)
    return cfg


def cmd_serve(args, extra):
    logging.basicConfig(level=getattr(logging, args.log_level.upper(), logging.INFO))
    from ..serve import launch_server

    cfg = _load(args, extra)
    restart = [s for s in (args.restart_stages or "").split(",") if s]
    launch_server(cfg, host=args.host, port=args.port, model_name=args.model_name, log_level=args.log_level,
                  restart_stages=restart)


def cmd_config(args, extra):
    import yaml

    cfg = _load(args, extra)
    if args.action == "view":
        print(yaml.safe_dump(cfg.model_dump(), sort_keys=False))
    else:
        if not args.output:
            raise SystemExit("config export needs --output")
        ConfigManager.to_file(cfg, args.output)
        print(f"wrote {args.output}")


def main(argv=None):
    ap = argparse.ArgumentParser(prog="sgl-omni")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("serve")
    s.add_argument("--model-path")
    s.add_argument("--config")
    s.add_argument("--text-only", action="store_true")
    s.add_argument("--host", default="0.0.0.0")
    s.add_argument("--port", type=int, default=8000)
    s.add_argument("--model-name")
    s.add_argument("--log-level", default="info")
    s.add_argument("--restart-stages", default="",
                   help="comma-separated stages whose process is restarted when it dies (multi-GPU placements)")
    c = sub.add_parser("config")
    c.add_argument("action", choices=["view", "export"])
    c.add_argument("--model-path")
    c.add_argument("--config")
    c.add_argument("--text-only", action="store_true")
    c.add_argument("--output")
    args, extra = ap.parse_known_args(argv)
    if args.cmd == "serve":
        cmd_serve(args, extra)
    else:
        cmd_config(args, extra)


if __name__ == "__main__":
    main(sys.argv[1:])
