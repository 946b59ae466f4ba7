"""mtorus.torch_ext"""
