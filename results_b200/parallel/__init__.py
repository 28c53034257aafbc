"""Collectives: communicator, native allreduce family, send/recv reference suite,
compressed collectives and weight transfer."""
