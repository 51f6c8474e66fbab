"""Utilities: GPU clock sampling, timing, logging, environment report."""
