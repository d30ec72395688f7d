"""Checker side of the test suite (CPU restatement + reference builds).

Test infrastructure only: the product package never imports this package.
"""
