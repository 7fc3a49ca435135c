"""Test infrastructure: the CPU checker (oracle.py) and the reference built from its sources (_ref/)."""
