"""Evaluation: protocol registry, runner with resume, parsers, graders, scoring, pull suite."""
