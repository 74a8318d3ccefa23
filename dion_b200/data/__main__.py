"""Inspect token files.

    python -m dion_b200.data info data/ [--seq-len 2048] [--decode-byte 200]

Per file: token count, bytes per token and header size; in total: tokens,
and windows of ``seq_len + 1`` tokens (what one epoch of the loader reads).
``--decode-byte N`` prints the first N tokens of the first file decoded with
the byte tokenizer.
"""
import argparse
import sys

import numpy as np

from . import expand_paths, token_file_info


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("command", choices=["info"])
    p.add_argument("paths", help="token files, directories or glob patterns (comma-separated)")
    p.add_argument("--seq-len", type=int, default=2048)
    p.add_argument("--bytes-per-token", type=int, default=0, help="for raw files without a header")
    p.add_argument("--decode-byte", type=int, default=0)
    a = p.parse_args(argv)
    files = expand_paths(a.paths)
    total = 0
    for f in files:
        info = token_file_info(f, a.bytes_per_token)
        total += info["tokens"]
        print(f"{f}: {info['tokens']:,} tokens, {info['bytes_per_token']} bytes/token, header {info['header_bytes']} B")
    print(f"total: {total:,} tokens in {len(files)} file(s); {total // (a.seq_len + 1):,} windows of "
          f"{a.seq_len + 1} tokens")
    if a.decode_byte and files:
        from .tokenize import ByteTokenizer

        info = token_file_info(files[0], a.bytes_per_token)
        dt = "<u2" if info["bytes_per_token"] == 2 else "<u4"
        ids = np.fromfile(files[0], dtype=dt, count=a.decode_byte, offset=info["header_bytes"]).tolist()
        print(repr(ByteTokenizer().decode(ids)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
