"""Golden vectors produced by the reference's own compiled code (make_golden.py)."""
