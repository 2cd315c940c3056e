"""Test infrastructure only: the CPU parity oracle for the LSTM + Linear path.

Imported by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline
leg.  The product package (persistent_lstm_hip_b200) never imports it.
"""
