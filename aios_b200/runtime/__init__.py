from .group import CandidateGroupRuntime, RoundResult

__all__ = ["CandidateGroupRuntime", "RoundResult"]
