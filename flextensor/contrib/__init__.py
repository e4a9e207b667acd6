"""Alias of :mod:`flextensor_b200.contrib`."""
