"""Native library loader and backend dispatch of the B200 MSDA build."""
