"""Candidate generation, planning, repair, selection and promotion."""
