"""mtorus.core"""
