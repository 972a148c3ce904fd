"""mxq.schedule — one float(e, m) per accumulator position of a reducer (mxq/schedule.py:21-53).

    load(path, rows=16)   CSV rows `position,e,m` or `position,B,e,m`, optional header
    fixed(e, m, rows=16)  [(e, m)] * rows
    HW_FINAL              the MX-Gemmini tapeout's 16 lanes: 8x e4m4, 2x e4m5, 5x e4m6, 1x bf16
"""
import csv
from pathlib import Path
from typing import List, Tuple, Union

__all__ = ["load", "fixed", "HW_FINAL"]

Entry = Tuple[int, int]

HW_FINAL: List[Entry] = [(4, 4)] * 8 + [(4, 5)] * 2 + [(4, 6)] * 5 + [(8, 7)]


def load(path: Union[str, Path], rows: int = 16) -> List[Entry]:
    """Read a schedule CSV: every position 0..rows-1 exactly once; a first row whose first cell is not a number
    is a header; rows of another width are skipped."""
    entries = {}
    with open(path) as f:
        reader = csv.reader(f)
        first = next(reader, None)
        body = ([first] if first and first[0].strip().isdigit() else []) + list(reader)
    for raw in body:
        cells = [c.strip() for c in raw if c.strip()]
        if len(cells) == 3:
            pos, e, m = (int(c) for c in cells)
        elif len(cells) == 4:
            pos, e, m = int(cells[0]), int(cells[2]), int(cells[3])
        else:
            continue
        if not 0 <= pos < rows:
            raise ValueError(f"schedule {path}: position {pos} outside 0..{rows - 1}")
        if pos in entries:
            raise ValueError(f"schedule {path}: position {pos} given twice")
        entries[pos] = (e, m)
    missing = [i for i in range(rows) if i not in entries]
    if missing:
        raise ValueError(f"schedule {path}: missing positions {missing}")
    return [entries[i] for i in range(rows)]


def fixed(e: int, m: int, rows: int = 16) -> List[Entry]:
    return [(e, m)] * rows
