#:set architecture = [('MaxPool', ['input'], [0, [0, 0, 0, 0], [3, 3]])]
#:set inputs = []
#:set trueInputs = [['input', [1, 2, 6, 6]]]
#:set outShape = [['output', [1, 2, 2, 2]]]
#:set outputs = {'output': 'input'}
