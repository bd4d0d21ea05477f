"""Puts the cb200 package (the parent of this directory) on sys.path so the
drop-in modules import the same way whether this directory or its parent is on
the path."""

import os
import sys

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if PKG_ROOT not in sys.path:
    sys.path.insert(0, PKG_ROOT)
