"""CPU oracle for the yanah_b200 decode path — TEST INFRASTRUCTURE ONLY.

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
use this package, as the checker / reported CPU baseline. The product
(``yanah_b200``) never imports it.
"""
