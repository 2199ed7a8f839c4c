"""Accuracy evaluation: teacher-forced scoring gates."""
