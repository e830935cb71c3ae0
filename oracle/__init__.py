"""TEST INFRASTRUCTURE ONLY: CPU restatements of the reference used as parity checkers."""
