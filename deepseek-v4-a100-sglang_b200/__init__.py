"""Package root: ``csrc/`` holds the sm_100a kernels and the C ABI,
``dsv4_b200/`` the Python host mirror of the reference operator API.
Add this directory to ``sys.path`` and ``import dsv4_b200``."""
