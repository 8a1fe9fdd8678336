"""Dataset and archive tools.

(reference: koochak/data/__main__.py:46-167)

    python -m koochak_b200.data archive SRC_DIR TARGET [--groups g.csv] [--exclude GLOB]...
    python -m koochak_b200.data pull COLLECTION DEST_DIR [--include GLOB]...
    python -m koochak_b200.data verify COLLECTION [--deep]
    python -m koochak_b200.data ls COLLECTION [--include GLOB] [--long]

Locations are paths or ``scheme://`` URIs resolved through the stores file
(``--stores`` or ``$KOOCHAK_STORES``). Reports print as JSON.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import sys
from typing import Optional, Sequence

from ..storage.archive import DEFAULT_PACK_BYTES, archive, load_file_list, pull, verify
from ..storage.collection import load_collection
from ..storage.store import open_store
from ..utils.sizes import parse_size


def _parser() -> argparse.ArgumentParser:
    common = argparse.ArgumentParser(add_help=False)
    common.add_argument("--stores", default=None, help="stores file (default: $KOOCHAK_STORES)")
    ap = argparse.ArgumentParser(prog="python -m koochak_b200.data", description="dataset and archive tools")
    sub = ap.add_subparsers(dest="command", required=True)
    a = sub.add_parser("archive", parents=[common], help="pack a local tree into a collection")
    a.add_argument("source", help="local directory")
    a.add_argument("target", help="collection location")
    a.add_argument("--groups", default=None, help="CSV with columns path,group[,order]")
    a.add_argument("--exclude", action="append", default=[], metavar="GLOB")
    a.add_argument("--include", action="append", default=[], metavar="GLOB")
    a.add_argument("--files-from", default=None, metavar="LIST", help="archive exactly these relative paths")
    a.add_argument("--layout", choices=("packed", "objects"), default="packed")
    a.add_argument("--pack-bytes", type=parse_size, default=DEFAULT_PACK_BYTES)
    a.add_argument("--object-bytes", type=parse_size, default=None)
    a.add_argument("--streams", type=int, default=None)
    a.add_argument("--skip-symlinks", action="store_true")
    a.add_argument("--min-age-hours", type=float, default=0.0)
    a.add_argument("--delete-source", action="store_true", help="delete sources after a deep verify passes")
    a.add_argument("--dry-run", action="store_true")
    p = sub.add_parser("pull", parents=[common], help="restore files from a collection")
    p.add_argument("source")
    p.add_argument("target")
    p.add_argument("--include", action="append", default=[], metavar="GLOB")
    p.add_argument("--streams", type=int, default=None)
    v = sub.add_parser("verify", parents=[common], help="check a collection")
    v.add_argument("location")
    v.add_argument("--deep", action="store_true")
    v.add_argument("--streams", type=int, default=None)
    ls = sub.add_parser("ls", parents=[common], help="list a collection's files")
    ls.add_argument("location")
    ls.add_argument("--include", action="append", default=[], metavar="GLOB")
    ls.add_argument("--long", action="store_true")
    return ap


def _local_root(location: str, stores: Optional[str]) -> str:
    st = open_store(location, stores_file=stores)
    root = getattr(st, "root", None)
    if root is None:
        raise SystemExit(f"archive sources must be local directories: {location}")
    return os.fspath(root)


def main(argv: Optional[Sequence[str]] = None) -> int:
    args = _parser().parse_args(argv)
    stores = args.stores
    if args.command == "archive":
        out = archive(_local_root(args.source, stores), open_store(args.target, stores_file=stores),
                      groups=args.groups, exclude=args.exclude, include=args.include or None,
                      files=load_file_list(args.files_from) if args.files_from else None, layout=args.layout,
                      pack_bytes=args.pack_bytes, object_bytes=args.object_bytes, streams=args.streams,
                      skip_symlinks=args.skip_symlinks, min_age_seconds=args.min_age_hours * 3600,
                      delete_sources=args.delete_source, dry_run=args.dry_run,
                      metadata={"source": args.source})
        if args.dry_run:
            print(json.dumps({"files": out.files, "packs": len(out.packs), "objects": len(out.objects),
                              "stored_bytes": out.stored_bytes}, indent=2, sort_keys=True))
        else:
            print(json.dumps({"packs_written": out.packs_written, "packs_reused": out.packs_reused,
                              "objects_copied": out.objects_copied, "bytes_read": out.bytes_read,
                              "files": len(out.collection.files), "deleted_files": out.deleted_files,
                              "manifest_sha256": out.collection.manifest_sha256, "seconds": out.seconds},
                             indent=2, sort_keys=True))
        return 0
    if args.command == "pull":
        rep = pull(open_store(args.source, stores_file=stores), open_store(args.target, stores_file=stores),
                   patterns=args.include, streams=args.streams)
        print(json.dumps(dataclasses.asdict(rep), indent=2, sort_keys=True))
        return 0
    if args.command == "verify":
        rep = verify(open_store(args.location, stores_file=stores), deep=args.deep, streams=args.streams)
        print(json.dumps(dataclasses.asdict(rep) | {"ok": rep.ok}, indent=2, sort_keys=True))
        return 0 if rep.ok else 1
    col = load_collection(open_store(args.location, stores_file=stores))
    for e in col.select(args.include):
        if not args.long:
            print(e.path)
        else:
            where = e.object if e.object is not None else f"{col.packs[e.pack].key}@{e.offset}"
            print(f"{e.size:>14} {e.sha256[:12]} {where} {e.path}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
