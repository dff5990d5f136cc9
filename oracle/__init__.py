"""CPU oracle package — TEST INFRASTRUCTURE ONLY (see oracle.cpp's header). Imported by tests/, by
__graft_entry__.smoke() and by bench.py's CPU-baseline leg; never by the product package."""
